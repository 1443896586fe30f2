// Shared device helpers for the sm_100a selective-scan kernels.
//
// Work decomposition used by every kernel here:
//   * one CTA owns one batch row b and a tile of 32 channels of one group (lane = channel);
//   * warp w owns states 4w .. 4w+3 of those channels, so a CTA has ceil(dstate/4)
//     warps (1, 2 or 4) for dstate <= 16; above that the states split into groups of 16,
//     one CTA (4 warps) per group, whose per-element partial sums meet in a workspace;
//   * time advances in tiles of kTile = 16 steps; each lane carries its 4 states in
//     registers across tiles, so the whole sequence is scanned without any cross-thread
//     scan (the reference runs a CUB block scan per state per 128-token chunk,
//     forward_kernel.cu:274-286);
//   * the forward writes the states at every tile boundary (the checkpoint buffer,
//     the counterpart of the reference's per-chunk carry x, forward_kernel.cu:171-172,
//     :285) so the backward can restart any tile without a second forward scan.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/mamba_b200_ss.h"

namespace ssb {

// Records e as the thread's last CUDA error (ss_last_cuda_error) and maps it to a status.
int record_cuda_status(cudaError_t e);
// Argument checks of a backward call (ss_capi.cu); own_states: f.ckpt and y not required.
int check_bwd(const ss_bwd_args* args, bool own_states);
// Raises the dynamic shared-memory limit of kernel `fn` to `smem` bytes (when above the 48 KB
// default) once per (device, kernel): setting the attribute on every launch costs host time.
cudaError_t ensure_smem_limit(const void* fn, size_t smem);


constexpr int kTile = 16;   // time steps per tile = checkpoint interval
constexpr int kCh = 32;     // channels per CTA (one per lane)
constexpr int kSPW = 4;     // states per warp
constexpr int kPad = 34;    // row stride (floats) of the [t][channel] partial-sum arrays
constexpr int kStages = 4;  // tiles of input in flight per CTA (TMA ring)
constexpr float kLog2e = 1.4426950408889634f;

// device status word codes (OR-ed into the caller-visible status buffer)
constexpr int kStatusTimeout = 1;   // a bounded wait on a TMA barrier gave up
// default limit of a bounded wait for a TMA tile (SM clock cycles, ~2 s at 1.9 GHz); a launch
// takes its limit from ss_set_wait_limit.  The drain after a timeout (waiting for the CTA's
// own copies still in flight before it exits) always uses the default.
constexpr long long kWaitCycles = 4000000000LL;

// ---- scalar conversions -----------------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f(T x);
template <> __device__ __forceinline__ float to_f<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <> __device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f(float x);
template <> __device__ __forceinline__ float from_f<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f<__half>(float x) { return __float2half_rn(x); }

template <typename T> __device__ __forceinline__ T zero_v() { return from_f<T>(0.f); }

// ---- transcendental helpers (hardware approximations, as the reference's fast-math build) --
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// ex2 kept in program order with the other ordered ex2 (asm volatile): a tile's block of
// independent decays is issued back to back ahead of the FMA chain that consumes it,
// instead of being sunk next to each use by the scheduler
__device__ __forceinline__ float ex2_ordered(float x) {
  float y;
  asm volatile("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fast_rcp(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2_fast(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// e^x via ex2 with a log2(e) prescale
__device__ __forceinline__ float exp_fast(float x) { return ex2(x * kLog2e); }
// 1 / (1 + e^-x)
__device__ __forceinline__ float sigmoid_fast(float x) { return fast_rcp(1.f + exp_fast(-x)); }
// log(1 + e) for e >= 0: the Taylor series e - e^2/2 + ... - e^6/6 below e = 1/16 (truncation
// error < e^7/7, i.e. < 1e-8 relative), log2(1 + e) * ln 2 above (where 1 + e carries no
// cancellation).  Replaces log1pf at a third of the instructions.
__device__ __forceinline__ float log1p_pos(float e) {
  float p = fmaf(e, -1.f / 6.f, 0.2f);
  p = fmaf(e, p, -0.25f);
  p = fmaf(e, p, 1.f / 3.f);
  p = fmaf(e, p, -0.5f);
  p = fmaf(e, p, 1.f);
  const float small = e * p;
  const float big = lg2_fast(1.f + e) * 0.69314718055994531f;
  return e < 0.0625f ? small : big;
}
// delta' = softplus(v) with the reference's threshold (forward_kernel.cu:216-221):
// log(1 + e^v) for v <= 20, v otherwise.
__device__ __forceinline__ float softplus_thr(float v) { return v <= 20.f ? log1p_pos(exp_fast(v)) : v; }
// softplus and its slope sigmoid(v) together (backward_kernel.cu:499-517): both from e = e^v
__device__ __forceinline__ void softplus_and_slope(float v, float& sp, float& slope) {
  const float e = exp_fast(v);
  const bool lin = v > 20.f;
  sp = lin ? v : log1p_pos(e);
  slope = lin ? 1.f : e * fast_rcp(1.f + e);
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization may
// start before the kernel ahead of it in the stream has finished.  griddep_wait() blocks until
// that kernel has completed and its writes are visible (it returns at once when the launch has no
// such dependency); griddep_launch_dependents() lets the next kernel of the stream start early.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// packed fp32x2 arithmetic (one instruction for two lanes of work on sm_100)
__device__ __forceinline__ float2 f2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }

// S consecutive shared-memory values of type T as floats (vector load when S*sizeof(T) is
// 8 or 16 bytes; the caller guarantees that alignment)
template <typename T, int S>
__device__ __forceinline__ void lds_run(const T* p, float (&v)[S]) {
  constexpr int BYTES = S * (int)sizeof(T);
  if constexpr (BYTES == 4 && sizeof(T) == 2) {
    union { uint32_t w; T e[2]; } u;
    u.w = *reinterpret_cast<const uint32_t*>(p);
    v[0] = to_f<T>(u.e[0]);
    v[1] = to_f<T>(u.e[1]);
  } else if constexpr (BYTES % 16 == 0 || BYTES == 8) {
    constexpr int CH = (BYTES % 16 == 0) ? 16 : 8;
    constexpr int PER = CH / (int)sizeof(T);
#pragma unroll
    for (int i = 0; i < S; i += PER) {
      union { uint4 q; uint2 d; T e[PER]; } u;
      if constexpr (CH == 16) u.q = *reinterpret_cast<const uint4*>(p + i);
      else u.d = *reinterpret_cast<const uint2*>(p + i);
#pragma unroll
      for (int k = 0; k < PER; ++k) v[i + k] = to_f<T>(u.e[k]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < S; ++i) v[i] = to_f<T>(p[i]);
  }
}

// ---- memory helpers -------------------------------------------------------------------
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
__device__ __forceinline__ void red_add_v2(float* p, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1,%2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void red_add(float* p, float a) { atomicAdd(p, a); }

// ---- mbarrier / TMA (cp.async.bulk.tensor) helpers ---------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// non-blocking probe of the phase `parity` (try_wait may suspend the thread for a while)
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for the phase `parity` of an mbarrier, giving up after `limit` SM clock cycles; a limit
// <= 0 only probes (non-blocking), so a tile that has not landed yet counts as a timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, long long limit) {
  if (limit <= 0) return mbar_test_wait(bar, parity);
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) return false;
  }
  return true;
}
// 3-D tiled TMA load global -> shared, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// Copy a (32 channels x kTile steps) tile of a (.., dim, seqlen) tensor into shared memory
// as dst[channel][t] (row-major, no padding).  Rows >= nrows and steps >= tlen read as 0.
// vec: the tile's rows start 16-byte aligned (checked on the host), so whole rows move as
// 16-byte vectors when the tile is full.
template <typename T, int NT>
__device__ __forceinline__ void load_tile(T (*dst)[kTile], const T* __restrict__ src, int64_t row_stride,
                                          int nrows, int tlen, bool vec) {
  constexpr int EPV = 16 / sizeof(T);  // elements per 16-byte vector
  constexpr int VPR = kTile / EPV;     // vectors per row
  if (vec && tlen == kTile) {
#pragma unroll
    for (int i = threadIdx.x; i < kCh * VPR; i += NT) {
      const int r = i / VPR, v = i % VPR;
      uint4 val = make_uint4(0u, 0u, 0u, 0u);
      if (r < nrows) val = ld_stream16(src + (int64_t)r * row_stride + v * EPV);
      *reinterpret_cast<uint4*>(&dst[r][v * EPV]) = val;
    }
  } else {
    for (int i = threadIdx.x; i < kCh * kTile; i += NT) {
      const int r = i / kTile, t = i % kTile;
      T val = zero_v<T>();
      if (r < nrows && t < tlen) val = src[(int64_t)r * row_stride + t];
      dst[r][t] = val;
    }
  }
}

// Copy the (dstate x kTile) slice of a variable B or C row block (stride seqlen between
// states) into dst[t][n] as fp32, zero-filled for n >= dstate or t >= tlen.
template <typename T, int NT, int NS>
__device__ __forceinline__ void load_bc_tile(float (*dst)[NS], const T* __restrict__ src, int64_t seqlen,
                                             int dstate, int tlen) {
  for (int i = threadIdx.x; i < NS * kTile; i += NT) {
    const int n = i / kTile, t = i % kTile;
    float v = 0.f;
    if (n < dstate && t < tlen) v = to_f<T>(src[(int64_t)n * seqlen + t]);
    dst[t][n] = v;
  }
}

// Per-element arrays of a tile ([32 channels][16 steps] as [channel][4 float4]), read by lane
// = channel, one float4 at a time.  With 2-byte I/O their rows are padded to kElemRow = 5 float4
// (80 bytes): "lane r reads float4 i of its row" then hits 8 distinct 16-byte bank groups per
// quarter warp, with no swizzle, so the address is a per-lane base plus a constant.  With 4-byte
// I/O the larger tiles leave no room for the pad (it would cost a CTA per SM), so the rows keep
// 4 float4 and float4 q of row r is stored at q ^ ((r >> 1) & 3), which makes the same reads
// conflict-free.
template <typename IT> constexpr int kElemRow = sizeof(IT) == 2 ? 5 : 4;
template <typename IT> __device__ __forceinline__ int erow(int r, int q) {
  return sizeof(IT) == 2 ? q : (q ^ ((r >> 1) & 3));
}

// Store S consecutive values of one row of a (.., dim, seqlen) tensor (S = 4, 8 or 16),
// vectorized when aligned and complete.
template <typename T, int S>
__device__ __forceinline__ void store_run(T* __restrict__ dst, const float (&v)[S], int nvalid, bool vec) {
  if constexpr (S * sizeof(T) == 4 && sizeof(T) == 2) {
    if (vec && nvalid == S) {
      union { uint32_t w; T e[2]; } pk;
      pk.e[0] = from_f<T>(v[0]);
      pk.e[1] = from_f<T>(v[1]);
      *reinterpret_cast<uint32_t*>(dst) = pk.w;
      return;
    }
  }
  if (vec && nvalid == S && (S * sizeof(T)) % 8 == 0) {
    if constexpr (S * sizeof(T) % 16 == 0) {
#pragma unroll
      for (int i = 0; i < S; i += 16 / sizeof(T)) {
        union { uint4 u; T e[16 / sizeof(T)]; } pk;
#pragma unroll
        for (int k = 0; k < 16 / (int)sizeof(T); ++k) pk.e[k] = from_f<T>(v[i + k]);
        *reinterpret_cast<uint4*>(dst + i) = pk.u;
      }
    } else {
#pragma unroll
      for (int i = 0; i < S; i += 8 / sizeof(T)) {
        union { uint2 u; T e[8 / sizeof(T)]; } pk;
#pragma unroll
        for (int k = 0; k < 8 / (int)sizeof(T); ++k) pk.e[k] = from_f<T>(v[i + k]);
        *reinterpret_cast<uint2*>(dst + i) = pk.u;
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < S; ++i)
      if (i < nvalid) dst[i] = from_f<T>(v[i]);
  }
}

// ---- element phases over (b, d, L) or (b, L, d) tiles ---------------------------------
// A tile of a per-element tensor arrives from TMA as [channel][step] for the (batch, dim,
// seqlen) layout (kBLD = false) and as [step][channel] for (batch, seqlen, dim) (kBLD = true).
// Element-phase thread (pc, pq) handles channel pc and steps pq*S .. pq*S + S - 1:
//   [channel][step] tiles: pc = tid / kNW, pq = tid % kNW — a channel's 16 steps are one
//     contiguous run, read with vector loads and stored as vectors;
//   [step][channel] tiles: pc = lane, pq = warp — a step's 32 channels are one contiguous run,
//     read by the 32 lanes together (one wavefront) and stored coalesced along the channels.
template <int kNW, bool kBLD> __device__ __forceinline__ int elem_pc(int tid) { return kBLD ? (tid & 31) : tid / kNW; }
template <int kNW, bool kBLD> __device__ __forceinline__ int elem_pq(int tid) { return kBLD ? (tid >> 5) : tid % kNW; }

// S consecutive steps of channel pc from a ring tile, as floats
template <typename IT, int S, bool kBLD>
__device__ __forceinline__ void lds_elems(const IT* tile, int pc, int pq, float (&v)[S]) {
  if constexpr (kBLD) {
#pragma unroll
    for (int i = 0; i < S; ++i) v[i] = to_f<IT>(tile[(pq * S + i) * kCh + pc]);
  } else {
    lds_run<IT, S>(tile + pc * kTile + pq * S, v);
  }
}

// Offset of (batch b, channel c, step 0) of a per-element tensor; consecutive steps are then
// step_stride<kBLD>(ds) elements apart (ds: the tensor's *_dim_stride field, which holds the
// seqlen stride for (b, L, d))
template <bool kBLD> __device__ __forceinline__ int64_t row_off(int64_t b, int64_t bs, int64_t c, int64_t ds) {
  return b * bs + c * (kBLD ? 1 : ds);
}
template <bool kBLD> __device__ __forceinline__ int64_t step_stride(int64_t ds) { return kBLD ? ds : 1; }

// Store S consecutive steps (from step t) of one channel's row
template <typename IT, int S, bool kBLD>
__device__ __forceinline__ void store_elems(IT* row, int64_t ds, int t, const float (&v)[S], int nvalid, bool vec) {
  if constexpr (kBLD) {
#pragma unroll
    for (int i = 0; i < S; ++i)
      if (i < nvalid) row[(int64_t)(t + i) * ds] = from_f<IT>(v[i]);
  } else {
    store_run<IT, S>(row + t, v, nvalid, vec);
  }
}

// Kernel-side parameter blocks (host fills the derived fields).  Tensor maps come first:
// CUtensorMap is 64-byte aligned.
struct FwdK {
  CUtensorMap tm_u, tm_d, tm_z, tm_B, tm_C;  // valid when the kernel is launched with TMA
  ss_fwd_args a;
  int dpg;        // channels per group
  int tpg;        // 32-channel tiles per group
  int nct;        // 32-channel tiles in all (ngroups * tpg)
  int nsg;        // state groups (1 for dstate <= 16, else ceil(dstate / 16))
  int ntiles;     // ceil(seqlen / kTile)
  int vec_u, vec_d, vec_z, vec_out, vec_y;
  int vec_work;   // workspace rows are 16-byte aligned (seqlen % 4 == 0)
  int* status;    // device status word (kStatus* bits), nullable
  long long wait_cycles;  // limit of a bounded wait for a TMA tile
  // time chunks (dstate <= 16, TMA path): the sequence splits into nchunk chunks of
  // chunk_tiles tiles, one CTA per (batch row, channel tile, chunk); chunk j's local end state
  // (from a zero state) is cstate[b][j][n][c] and its sum of delta' csum[b][j][c], both written
  // by ss_fwd_chunk_kernel for j < nchunk - 1 (pointers into the caller's workspace)
  int nchunk, chunk_tiles;
  float* cstate;
  float* csum;
};

struct BwdK {
  CUtensorMap tm_u, tm_d, tm_z, tm_g, tm_y, tm_B, tm_C, tm_h;
  ss_bwd_args a;
  int dpg, tpg, nct, nsg, ntiles;
  int vec_u, vec_d, vec_z, vec_dout, vec_du, vec_dd, vec_dz, vec_y;
  int vec_dbc;    // dB/dC rows are 16-byte aligned (seqlen % 4 == 0)
  int* status;
  long long wait_cycles;
  // time chunks, as in FwdK: chunk j's local carry into the step before it (the reverse
  // recurrence run over the chunk from a zero carry) is ccarry[b][j][n][c] and its sum of
  // delta' csum[b][j][c], both written by ss_bwd_carry_kernel for j >= 1
  int nchunk, chunk_tiles;
  float* ccarry;
  float* csum;
  // 1: launched as a programmatic dependent of the kernel that zeroes dA / dB / dC / dD /
  // ddelta_bias (whole rows, no state groups), so the kernel waits for it before its tile loop
  // (its setup and first copies overlap that kernel); the time-chunked launch follows the carry
  // pass, which starts only after that zeroing has completed
  int zero_dep;
};

constexpr int kGroupStates = 16;  // states per CTA when dstate > 16 (4 warps x 4)
inline int state_groups(int dstate) { return dstate <= kGroupStates ? 1 : (dstate + kGroupStates - 1) / kGroupStates; }

}  // namespace ssb
