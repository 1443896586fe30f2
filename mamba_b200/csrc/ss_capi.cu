// C ABI of libmamba_b200_ss.so: argument validation, derived launch parameters and
// dtype dispatch.  The reference has no input checks at all (its binding,
// csrc/selective_scan/selective_scan.cpp:184-329, passes raw pointers straight through);
// here every call is checked first and reports a status code instead of faulting.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <cmath>
#include <mutex>
#include <unordered_map>

#include "../../include/mamba_b200_ss.h"
#include "ss_common.cuh"
#include "ss_step.cuh"  // step_shape

namespace ssb {
template <typename IT> cudaError_t launch_fwd(const FwdK&, cudaStream_t, bool);
template <typename IT> cudaError_t launch_bwd(const BwdK&, cudaStream_t, bool);
template <typename IT> cudaError_t launch_step(const ss_step_args&, cudaStream_t);
}  // namespace ssb

namespace ssb {
// Zeroes up to 5 fp32 spans (the backward's summed gradients) before the backward runs.  It
// releases its programmatic dependents at once: the backward launched after it starts (setup,
// first tile copies) while these stores run, and waits for this grid (griddep_wait) before its
// tile loop.
struct ZeroSpans {
  float* p[5];
  long long n[5];
  int k;
};

__global__ void __launch_bounds__(256) zero_spans_kernel(const __grid_constant__ ZeroSpans z) {
  griddep_launch_dependents();
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (int s = 0; s < z.k; ++s) {
    float* p = z.p[s];
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < z.n[s]; i += stride) p[i] = 0.f;
  }
}

cudaError_t launch_zero_spans(const ZeroSpans& z, cudaStream_t st) {
  long long total = 0;
  for (int s = 0; s < z.k; ++s) total += z.n[s];
  if (total == 0) return cudaSuccess;
  const long long blocks = std::min<long long>((total + 255) / 256, 2 * 148);
  zero_spans_kernel<<<(unsigned)blocks, 256, 0, st>>>(z);
  return cudaGetLastError();
}
}  // namespace ssb

// One status word per device that loads the library: kernels OR kStatus* bits into it when
// a bounded wait gives up (see ss_device_status).
__device__ int g_ss_status;

namespace {
thread_local int g_last_cuda = 0;
// limit of the kernels' bounded waits for a TMA tile, for launches from this process
std::atomic<long long> g_wait_cycles{ssb::kWaitCycles};
// time chunks per scan pass: 0 chooses them from the shape (chunk_count below)
std::atomic<int> g_time_chunks{0};
}  // namespace

// shared with the other translation units of the library (hidden visibility)
int ssb::record_cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return SS_OK;
  g_last_cuda = (int)e;
  return SS_ERR_CUDA;
}

namespace {

int* status_ptr() {
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, g_ss_status) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  return static_cast<int*>(p);
}

// cuTensorMapEncodeTiled from the driver, fetched through the runtime (no -lcuda link)
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

CUtensorMapDataType tm_type(int dt) {
  return dt == SS_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                      : (dt == SS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
}

// 3-D tiled map: extents (d0 innermost, d1, d2), byte strides of d1 and d2, box (b0, b1, 1).
// Returns false when TMA cannot describe the tensor (alignment), so the caller falls back.
bool map3(CUtensorMap* m, const void* base, int dt, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
          uint64_t s2, uint32_t b0, uint32_t b1) {
  auto fn = encode_fn();
  const uint64_t es = dt == SS_F32 ? 4 : 2;
  if (fn == nullptr || base == nullptr || (reinterpret_cast<uintptr_t>(base) & 15) || (s1 & 15) || (s2 & 15) ||
      ((b0 * es) & 15) || s1 >= (1ull << 40) || s2 >= (1ull << 40))
    return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(m, tm_type(dt), 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A per-element tensor -> box of 16 steps x 32 channels.  (batch, dim, seqlen) layout: extents
// (seqlen, dim, batch), ds = dim stride; (batch, seqlen, dim) layout: extents (dim, seqlen,
// batch), ds = seqlen stride (the box lands as [step][channel]).
bool map_rows(CUtensorMap* m, const void* p, int dt, const ss_fwd_args& a, int64_t bs, int64_t ds) {
  const uint64_t es = dt == SS_F32 ? 4 : 2;
  if (ds < 0 || bs < 0) return false;
  if (a.layout == SS_LAYOUT_BLD) {
    const uint64_t s1 = a.seqlen > 1 ? (uint64_t)ds * es : (uint64_t)a.dim * es;
    const uint64_t s2 = a.batch > 1 ? (uint64_t)bs * es : s1 * (uint64_t)a.seqlen;
    return map3(m, p, dt, (uint64_t)a.dim, (uint64_t)a.seqlen, (uint64_t)a.batch, s1, s2, ssb::kCh, ssb::kTile);
  }
  const uint64_t s1 = a.dim > 1 ? (uint64_t)ds * es : (uint64_t)a.seqlen * es;
  const uint64_t s2 = a.batch > 1 ? (uint64_t)bs * es : s1 * (uint64_t)a.dim;
  return map3(m, p, dt, (uint64_t)a.seqlen, (uint64_t)a.dim, (uint64_t)a.batch, s1, s2, ssb::kTile, ssb::kCh);
}

// (batch, seqlen, dim) calls: every tile's first channel (the tensor maps' innermost
// coordinate) must start 16 bytes apart, i.e. the channels of a group must span whole 16-byte
// units when there are several groups
bool bld_channels_aligned(const ss_fwd_args& a) {
  const int64_t dpg = a.dim / a.ngroups;
  const int64_t es = a.io_dtype == SS_F32 ? 4 : 2;
  return a.ngroups == 1 || (dpg * es) % 16 == 0;
}

// variable B / C (batch, ngroups, dstate, seqlen) -> box of 16 steps x (padded) dstate
bool map_bc(CUtensorMap* m, const void* p, const ss_fwd_args& a) {
  const uint64_t es = a.bc_dtype == SS_F32 ? 4 : 2;
  const uint32_t ns = 4u * (uint32_t)(a.dstate <= 4 ? 1 : (a.dstate <= 8 ? 2 : 4));
  return map3(m, p, a.bc_dtype, (uint64_t)a.seqlen, (uint64_t)a.dstate, (uint64_t)a.batch * a.ngroups,
              (uint64_t)a.seqlen * es, (uint64_t)a.seqlen * a.dstate * es, ssb::kTile, ns);
}

int cuda_status(cudaError_t e) { return ssb::record_cuda_status(e); }


size_t esize(int dt) { return dt == SS_F32 ? 4 : 2; }
bool dtype_ok(int dt) { return dt == SS_F32 || dt == SS_BF16 || dt == SS_F16; }

// every (batch, channel) row of a (batch, dim, seqlen) view starts 16-byte aligned
bool rows16(const void* p, int64_t bs, int64_t ds, size_t es) {
  return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && ((bs * (int64_t)es) & 15) == 0 &&
         ((ds * (int64_t)es) & 15) == 0;
}

constexpr int64_t kMaxGrid = 2147483647;  // gridDim.x

int check_fwd(const ss_fwd_args* a) {
  if (a == nullptr) return SS_ERR_INVALID;
  if (a->batch < 0 || a->dim < 1 || a->seqlen < 0 || a->dstate < 1 || a->ngroups < 1) return SS_ERR_INVALID;
  if (a->dim % a->ngroups != 0) return SS_ERR_INVALID;
  if (a->dstate > SS_MAX_DSTATE) return SS_ERR_UNSUPPORTED;
  // flattened grids: scan CTAs (batch x state groups x 32-channel tiles) and, with state
  // groups, the finishing pass (batch x dim x 256-step chunks)
  const int64_t dpg = a->dim / a->ngroups;
  const int64_t nct = (int64_t)a->ngroups * ((dpg + ssb::kCh - 1) / ssb::kCh);
  const int64_t nsg = ssb::state_groups(a->dstate);
  if ((int64_t)a->batch * nsg * nct > kMaxGrid) return SS_ERR_UNSUPPORTED;
  if (nsg > 1) {
    if ((int64_t)a->batch * a->dim * (((int64_t)a->seqlen + 255) / 256) > kMaxGrid) return SS_ERR_UNSUPPORTED;
    if (a->work == nullptr && a->batch > 0 && a->seqlen > 0) return SS_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(a->work) & 15) != 0) return SS_ERR_INVALID;  // vector reductions
  }
  if (!dtype_ok(a->io_dtype) || !dtype_ok(a->bc_dtype)) return SS_ERR_UNSUPPORTED;
  if (a->bc_dtype != SS_F32 && a->bc_dtype != a->io_dtype) return SS_ERR_UNSUPPORTED;
  if (a->layout != SS_LAYOUT_BDL && a->layout != SS_LAYOUT_BLD) return SS_ERR_INVALID;
  if (a->layout == SS_LAYOUT_BLD && (nsg > 1 || !bld_channels_aligned(*a))) return SS_ERR_UNSUPPORTED;
  // empty (batch, dim, seqlen) tensors may carry null data pointers; A and constant B / C never are empty
  const bool empty = a->batch == 0 || a->seqlen == 0;
  if (!a->A || (!a->var_B && !a->B) || (!a->var_C && !a->C)) return SS_ERR_INVALID;
  if (!empty && (!a->u || !a->delta || !a->B || !a->C)) return SS_ERR_INVALID;
  if (a->u_batch_stride < 0 || a->u_dim_stride < 0 || a->delta_batch_stride < 0 || a->delta_dim_stride < 0)
    return SS_ERR_INVALID;
  if (a->z && (a->z_batch_stride < 0 || a->z_dim_stride < 0)) return SS_ERR_INVALID;
  return SS_OK;
}

template <typename K>
void derive(const ss_fwd_args& a, K& P) {
  P.dpg = a.dim / a.ngroups;
  P.tpg = (P.dpg + ssb::kCh - 1) / ssb::kCh;
  P.nct = a.ngroups * P.tpg;
  P.nsg = ssb::state_groups(a.dstate);
  P.ntiles = (a.seqlen + ssb::kTile - 1) / ssb::kTile;
  P.nchunk = 1;  // one chunk: the whole sequence (set_chunks may split it)
  P.chunk_tiles = P.ntiles;
}

// ---- time chunks.  A scan pass runs one CTA per (batch row, 32-channel tile); when that grid
// cannot fill the GPU the sequence is cut into chunks (ss_chunk.cuh), which costs a summary
// pass over all but one chunk (about half a forward, a fifth of a backward) and buys
// parallelism.  The count minimises a wave model of the pass:
//     time(K) ~ ceil(ctas K / slots) / K * (1 + extra (K - 1) / K)
// (slots = SMs x CTAs resident per SM): its minimum, used only when the model gains >= 15 %.
// Measured on a B200 (forced counts): the forward of batch 2 x 1536 channels x 2048 steps
// takes 0.177 ms whole and 0.10 ms at 4 - 16 chunks; batch 1 x 5120 x 32768 steps 3.29 ms
// whole and 1.95 - 2.03 ms at 8 - 48 chunks; batch 8 x 1536 x 2048 (384 CTAs) is slower split.
constexpr int kSMs = 148;            // B200
constexpr int kMinChunkTiles = 8;    // >= 128 steps per chunk
constexpr int kMaxChunks = 64;

int chunk_count(int64_t ctas, int ntiles, int ctas_per_sm, double extra) {
  const int forced = g_time_chunks.load(std::memory_order_relaxed);
  if (forced > 0) return std::max(1, std::min(forced, ntiles));
  const int kmax = (int)std::min<int64_t>(kMaxChunks, ntiles / kMinChunkTiles);
  if (kmax < 2 || ctas <= 0) return 1;
  const double slots = (double)kSMs * ctas_per_sm;
  double tmin = 1.0;
  int best = 1;
  for (int k = 2; k <= kmax; ++k) {
    const double t = std::ceil((double)ctas * k / slots) / k * (1.0 + extra * (k - 1) / k);
    if (t < tmin) {
      tmin = t;
      best = k;
    }
  }
  return tmin > 0.85 ? 1 : best;
}

int64_t channel_tiles(int dim, int ngroups) {
  const int64_t dpg = dim / ngroups;
  return (int64_t)ngroups * ((dpg + ssb::kCh - 1) / ssb::kCh);
}
// forward: 4 CTAs per SM; its chunk pass costs about half the forward
int fwd_chunk_count(int batch, int64_t nct, int ntiles) { return chunk_count((int64_t)batch * nct, ntiles, 4, 0.5); }
// backward: 3 CTAs per SM; its carry pass costs about a fifth of the backward
int bwd_chunk_count(int batch, int64_t nct, int ntiles) { return chunk_count((int64_t)batch * nct, ntiles, 3, 0.2); }
// chunks the workspace of ss_work_elems holds (the larger pass, channel tiles of one group)
int sized_chunks(int batch, int dim, int seqlen, int dstate) {
  if (batch <= 0 || dim <= 0 || seqlen <= 0 || dstate > ssb::kGroupStates) return 1;
  const int ntiles = (seqlen + ssb::kTile - 1) / ssb::kTile;
  const int64_t nct = channel_tiles(dim, 1);
  return std::max(fwd_chunk_count(batch, nct, ntiles), bwd_chunk_count(batch, nct, ntiles));
}

// Splits a pass into chunks when the workspace allows: K from `want`, capped by what the
// workspace holds; chunk_tiles such that no chunk is empty.  Returns the chunk count.
template <typename K>
int set_chunks(K& P, int want, const ss_fwd_args& a) {
  P.nchunk = 1;
  P.chunk_tiles = P.ntiles;
  const int64_t ctas = std::max<int64_t>(1, (int64_t)a.batch * P.nct);
  const int k = (int)std::min<int64_t>(std::min(want, sized_chunks(a.batch, a.dim, a.seqlen, a.dstate)),
                                       kMaxGrid / ctas);
  if (k <= 1 || a.work == nullptr || P.nsg != 1) return 1;
  P.chunk_tiles = (P.ntiles + k - 1) / k;
  P.nchunk = (P.ntiles + P.chunk_tiles - 1) / P.chunk_tiles;
  return P.nchunk;
}

template <typename F>
int dispatch(int io, F&& f) {
  switch (io) {
    case SS_F32: return cuda_status(f(float{}));
    case SS_BF16: return cuda_status(f(__nv_bfloat16{}));
    case SS_F16: return cuda_status(f(__half{}));
    default: return SS_ERR_UNSUPPORTED;
  }
}

}  // namespace

cudaError_t ssb::ensure_smem_limit(const void* fn, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  static std::mutex mu;
  static std::unordered_map<const void*, std::array<size_t, 64>> done;  // limit set, per device
  if (dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lock(mu);
    if (done[fn][dev] >= smem) return cudaSuccess;
  }
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess && dev >= 0 && dev < 64) {
    std::lock_guard<std::mutex> lock(mu);
    done[fn][dev] = std::max(done[fn][dev], smem);
  }
  return e;
}

// Argument checks of a backward call (shared with ss_bwd_noalloc, which makes them before it
// launches anything).  own_states: the caller recomputes the forward's states and ungated
// output itself, so f.ckpt and y are not required.
int ssb::check_bwd(const ss_bwd_args* args, bool own_states) {
  if (args == nullptr) return SS_ERR_INVALID;
  const ss_fwd_args& f = args->f;
  int rc = check_fwd(&f);
  if (rc != SS_OK) return rc;
  // with no batch rows or no steps the (batch, dim, seqlen) tensors and variable dB / dC are empty
  const bool empty = f.batch == 0 || f.seqlen == 0;
  if (!args->dA || (!f.var_B && !args->dB) || (!f.var_C && !args->dC)) return SS_ERR_INVALID;
  if (!empty && (!args->dout || !args->du || !args->ddelta || !args->dB || !args->dC)) return SS_ERR_INVALID;
  if (f.z && !empty && (!args->dz || (!own_states && !args->y))) return SS_ERR_INVALID;
  if (!own_states && !f.ckpt && f.seqlen > kTile && f.batch > 0) return SS_ERR_INVALID;
  if (args->dout_batch_stride < 0 || args->dout_dim_stride < 0 || args->du_batch_stride < 0 ||
      args->du_dim_stride < 0 || args->ddelta_batch_stride < 0 || args->ddelta_dim_stride < 0)
    return SS_ERR_INVALID;
  if (f.z && (args->dz_batch_stride < 0 || args->dz_dim_stride < 0 ||
              (!own_states && (args->y_batch_stride < 0 || args->y_dim_stride < 0))))
    return SS_ERR_INVALID;
  return SS_OK;
}

extern "C" {

size_t ss_ckpt_elems(int batch, int dim, int seqlen, int dstate) {
  if (batch <= 0 || dim <= 0 || seqlen <= 0 || dstate <= 0) return 0;
  const size_t ntiles = ((size_t)seqlen + ssb::kTile - 1) / ssb::kTile;
  return (size_t)batch * ntiles * (size_t)dstate * (size_t)dim;
}

size_t ss_work_elems(int batch, int dim, int seqlen, int dstate) {
  if (batch <= 0 || dim <= 0 || seqlen <= 0) return 0;
  if (dstate > ssb::kGroupStates) return 2 * (size_t)batch * (size_t)dim * (size_t)seqlen;
  // time chunks: per chunk a state (or carry) per (channel, state) and a sum of delta' per channel
  const int k = sized_chunks(batch, dim, seqlen, dstate);
  return k > 1 ? (size_t)batch * k * ((size_t)dstate + 1) * (size_t)dim : 0;
}

int ss_fwd(const ss_fwd_args* args, void* stream) {
  int rc = check_fwd(args);
  if (rc != SS_OK) return rc;
  if (args->out_batch_stride < 0 || args->out_dim_stride < 0) return SS_ERR_INVALID;
  if (args->batch == 0) return SS_OK;
  if (!args->out && args->seqlen > 0) return SS_ERR_INVALID;
  if (args->seqlen == 0) {  // no steps: the final state is the zero initial state
    if (args->last_state == nullptr) return SS_OK;
    const size_t bytes = (size_t)args->batch * args->dim * args->dstate * sizeof(float);
    return cuda_status(cudaMemsetAsync(args->last_state, 0, bytes, (cudaStream_t)stream));
  }
  ssb::FwdK P{};
  P.a = *args;
  derive(P.a, P);
  const size_t es = esize(args->io_dtype);
  P.vec_u = rows16(args->u, args->u_batch_stride, args->u_dim_stride, es);
  P.vec_d = rows16(args->delta, args->delta_batch_stride, args->delta_dim_stride, es);
  P.vec_z = args->z ? rows16(args->z, args->z_batch_stride, args->z_dim_stride, es) : 0;
  P.vec_out = rows16(args->out, args->out_batch_stride, args->out_dim_stride, es);
  P.vec_y = args->out_y ? rows16(args->out_y, args->out_y_batch_stride, args->out_y_dim_stride, es) : 0;
  P.vec_work = args->work != nullptr && (reinterpret_cast<uintptr_t>(args->work) & 15) == 0 && (args->seqlen % 4) == 0;
  P.status = status_ptr();
  P.wait_cycles = g_wait_cycles.load(std::memory_order_relaxed);
  const ss_fwd_args& a = *args;
  bool tma = map_rows(&P.tm_u, a.u, a.io_dtype, a, a.u_batch_stride, a.u_dim_stride) &&
             map_rows(&P.tm_d, a.delta, a.io_dtype, a, a.delta_batch_stride, a.delta_dim_stride);
  if (tma && a.z) tma = map_rows(&P.tm_z, a.z, a.io_dtype, a, a.z_batch_stride, a.z_dim_stride);
  if (tma && a.var_B) tma = map_bc(&P.tm_B, a.B, a);
  if (tma && a.var_C) tma = map_bc(&P.tm_C, a.C, a);
  if (!tma && a.layout == SS_LAYOUT_BLD) return SS_ERR_UNSUPPORTED;  // (b, L, d) tiles need tensor maps
  if (tma && set_chunks(P, fwd_chunk_count(a.batch, P.nct, P.ntiles), a) > 1) {
    P.cstate = a.work;
    P.csum = a.work + (size_t)a.batch * P.nchunk * a.dstate * (size_t)a.dim;
  }
  cudaStream_t st = (cudaStream_t)stream;
  return dispatch(args->io_dtype, [&](auto tag) { return ssb::launch_fwd<decltype(tag)>(P, st, tma); });
}

int ss_bwd(const ss_bwd_args* args, void* stream) {
  int rc = ssb::check_bwd(args, false);
  if (rc != SS_OK) return rc;
  const ss_fwd_args& f = args->f;
  cudaStream_t st = (cudaStream_t)stream;
  // accumulated outputs start from zero (zeroed once the call is known to run)
  // the summed gradients, as runs of buffers that lie end to end (the Python layer allocates
  // dA / dD / ddelta_bias and dB / dC so): one memset, or one span of the zeroing kernel, per run
  ssb::ZeroSpans zs{};
  {
    const size_t nA = (size_t)f.dim * f.dstate;
    const size_t nBv = (size_t)f.batch * f.ngroups * f.dstate * (size_t)f.seqlen;
    const size_t nB = f.var_B ? nBv : nA, nC = f.var_C ? nBv : nA;
    auto add = [&](float* ptr, size_t elems) {
      if (ptr == nullptr || elems == 0) return;
      if (zs.k > 0 && zs.p[zs.k - 1] + zs.n[zs.k - 1] == ptr) zs.n[zs.k - 1] += (long long)elems;
      else { zs.p[zs.k] = ptr; zs.n[zs.k] = (long long)elems; ++zs.k; }
    };
    add(args->dA, nA);
    add(args->dD, f.dim);
    add(args->ddelta_bias, f.dim);
    add(args->dB, nB);
    add(args->dC, nC);
  }
  auto zero_sums = [&]() {
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < zs.k && e == cudaSuccess; ++i) e = cudaMemsetAsync(zs.p[i], 0, zs.n[i] * sizeof(float), st);
    return e;
  };
  if (f.batch == 0 || f.seqlen == 0) return cuda_status(zero_sums());
  ssb::BwdK P{};
  P.a = *args;
  derive(f, P);
  const size_t es = esize(f.io_dtype);
  P.vec_u = rows16(f.u, f.u_batch_stride, f.u_dim_stride, es);
  P.vec_d = rows16(f.delta, f.delta_batch_stride, f.delta_dim_stride, es);
  P.vec_z = f.z ? rows16(f.z, f.z_batch_stride, f.z_dim_stride, es) : 0;
  P.vec_dout = rows16(args->dout, args->dout_batch_stride, args->dout_dim_stride, es);
  P.vec_du = rows16(args->du, args->du_batch_stride, args->du_dim_stride, es);
  P.vec_dd = rows16(args->ddelta, args->ddelta_batch_stride, args->ddelta_dim_stride, es);
  P.vec_dz = f.z ? rows16(args->dz, args->dz_batch_stride, args->dz_dim_stride, es) : 0;
  P.vec_y = f.z ? rows16(args->y, args->y_batch_stride, args->y_dim_stride, es) : 0;
  P.vec_dbc = (f.seqlen % 4) == 0 && (reinterpret_cast<uintptr_t>(args->dB) & 15) == 0 &&
              (reinterpret_cast<uintptr_t>(args->dC) & 15) == 0;
  P.status = status_ptr();
  P.wait_cycles = g_wait_cycles.load(std::memory_order_relaxed);
  // the checkpoint tile starts at channel c0: TMA needs c0 * 4 bytes to be 16-byte aligned;
  // the TMA ring stages B / C in the I/O dtype
  bool tma = (f.ngroups == 1 || (P.dpg % 4) == 0) && (f.bc_dtype == f.io_dtype || (!f.var_B && !f.var_C)) &&
             map_rows(&P.tm_u, f.u, f.io_dtype, f, f.u_batch_stride, f.u_dim_stride) &&
             map_rows(&P.tm_d, f.delta, f.io_dtype, f, f.delta_batch_stride, f.delta_dim_stride) &&
             map_rows(&P.tm_g, args->dout, f.io_dtype, f, args->dout_batch_stride, args->dout_dim_stride);
  if (tma && f.z)
    tma = map_rows(&P.tm_z, f.z, f.io_dtype, f, f.z_batch_stride, f.z_dim_stride) &&
          map_rows(&P.tm_y, args->y, f.io_dtype, f, args->y_batch_stride, args->y_dim_stride);
  if (tma && f.var_B) tma = map_bc(&P.tm_B, f.B, f);
  if (tma && f.var_C) tma = map_bc(&P.tm_C, f.C, f);
  if (tma && f.ckpt) {
    const uint32_t ns = 4u * (uint32_t)(f.dstate <= 4 ? 1 : (f.dstate <= 8 ? 2 : 4));
    tma = map3(&P.tm_h, f.ckpt, SS_F32, (uint64_t)f.dim, (uint64_t)f.dstate, (uint64_t)f.batch * P.ntiles,
               (uint64_t)f.dim * 4, (uint64_t)f.dim * f.dstate * 4, ssb::kCh, ns);
  } else if (tma && P.ntiles > 1) {
    tma = false;
  }
  if (!tma && f.layout == SS_LAYOUT_BLD) return SS_ERR_UNSUPPORTED;  // (b, L, d) tiles need tensor maps
  if (tma && set_chunks(P, bwd_chunk_count(f.batch, P.nct, P.ntiles), f) > 1) {
    P.ccarry = f.work;
    P.csum = f.work + (size_t)f.batch * P.nchunk * f.dstate * (size_t)f.dim;
  }
  cudaError_t e;
  if (P.nsg > 1) {
    e = zero_sums();
  } else {
    // our zeroing kernel lets the backward start before it ends (programmatic dependent launch);
    // whole-row launches wait for it before their tile loop, time-chunked ones need not (the
    // carry pass between them starts only after it has completed)
    e = ssb::launch_zero_spans(zs, st);
    P.zero_dep = (P.nchunk == 1 && zs.k > 0) ? 1 : 0;  // (dA is never empty: the kernel ran)
  }
  if (e != cudaSuccess) return cuda_status(e);
  return dispatch(f.io_dtype, [&](auto tag) { return ssb::launch_bwd<decltype(tag)>(P, st, tma); });
}

int ss_step(const ss_step_args* a, void* stream) {
  if (a == nullptr) return SS_ERR_INVALID;
  if (a->batch < 0 || a->dim < 1 || a->dstate < 1 || a->ngroups < 1 || a->dim % a->ngroups) return SS_ERR_INVALID;
  if (a->dstate > SS_MAX_DSTATE) return SS_ERR_UNSUPPORTED;
  {
    int tpc, chunks;
    ssb::step_shape(a->dstate, tpc, chunks);
    const int64_t cpb = 128 / tpc;
    if ((int64_t)a->batch * ((a->dim + cpb - 1) / cpb) > kMaxGrid) return SS_ERR_UNSUPPORTED;
  }
  if (!dtype_ok(a->io_dtype) || !dtype_ok(a->bc_dtype)) return SS_ERR_UNSUPPORTED;
  if (a->bc_dtype != SS_F32 && a->bc_dtype != a->io_dtype) return SS_ERR_UNSUPPORTED;
  if (!a->A || a->B_batch_stride < 0 || a->C_batch_stride < 0) return SS_ERR_INVALID;
  if (a->dt_proj && (a->dt_rank < 1 || a->dt_rank > 1024)) return a->dt_rank < 1 ? SS_ERR_INVALID : SS_ERR_UNSUPPORTED;
  if (a->batch == 0) return SS_OK;  // the per-sequence tensors are empty and may carry null pointers
  if (!a->state || !a->x || !a->dt || !a->B || !a->C || !a->out) return SS_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  return dispatch(a->io_dtype, [&](auto tag) { return ssb::launch_step<decltype(tag)>(*a, st); });
}

const char* ss_status_string(int s) {
  switch (s) {
    case SS_OK: return "ok";
    case SS_ERR_INVALID: return "invalid argument (null pointer, size, stride or group count)";
    case SS_ERR_UNSUPPORTED: return "unsupported dtype combination, dstate > 256 or a size beyond the launch grid";
    case SS_ERR_CUDA: return "CUDA runtime error (see ss_last_cuda_error)";
    default: return "unknown status";
  }
}

int ss_last_cuda_error(void) { return g_last_cuda; }

int ss_abi_version(void) { return SS_ABI_VERSION; }

int ss_set_time_chunks(int chunks) { return g_time_chunks.exchange(chunks > 0 ? chunks : 0); }

long long ss_set_wait_limit(long long cycles) {
  return g_wait_cycles.exchange(cycles < 0 ? ssb::kWaitCycles : cycles);
}

int ss_device_status(int reset, void* stream) {
  int* p = status_ptr();
  if (p == nullptr) return -1;
  int v = 0;
  cudaStream_t st = (cudaStream_t)stream;
  if (cudaMemcpyAsync(&v, p, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess) return -1;
  if (reset && cudaMemsetAsync(p, 0, sizeof(int), st) != cudaSuccess) return -1;
  if (cudaStreamSynchronize(st) != cudaSuccess) return -1;
  return v;
}

size_t ss_struct_size(int which) {
  switch (which) {
    case 0: return sizeof(ss_fwd_args);
    case 1: return sizeof(ss_bwd_args);
    case 2: return sizeof(ss_step_args);
    case 3: return sizeof(ss_conv_args);
    case 4: return sizeof(ss_conv_bwd_args);
    case 5: return sizeof(ss_conv_step_args);
    case 6: return sizeof(ss_rmsnorm_args);
    case 7: return sizeof(ss_rmsnorm_bwd_args);
    case 8: return sizeof(ss_mamba_step_args);
    default: return 0;
  }
}

}  // extern "C"
