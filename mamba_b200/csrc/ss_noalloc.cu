// ss_bwd_noalloc: the backward scan for callers that cannot allocate device memory.
//
// ss_bwd needs the forward's state buffer (ckpt).  A caller that kept it can use ss_bwd;
// a caller that did not keep it and cannot allocate one — for example an FFI binding from a
// language with no CUDA allocator of its own, or a serving process whose device memory is
// entirely owned by its own pool, where cudaMalloc would fail or would synchronise the
// device in the middle of a step — calls this entry point instead.  It recomputes the states
// into a scratch array that lives in this library (a file-scope __device__ array, one per
// GPU that loads the library, held until the process exits) and then runs the backward.
// It calls no cudaMalloc / cudaFree and no allocating library routine.
//
// Limits and behaviour:
//   * the state buffer must fit: ss_ckpt_elems(batch, dim, seqlen, dstate) must be at most
//     SS_NOALLOC_MAX_CKPT_ELEMS (4 Mi floats, 16 MiB); larger calls return
//     SS_ERR_UNSUPPORTED before touching the device;
//   * every argument is checked before anything is launched, so a rejected call leaves du and
//     dz untouched;
//   * the scratch array's device address is looked up (set-up) on the first call with a given
//     device and CUDA context current, and again whenever the current context changes (a
//     device reset, another driver context) or a launch through it failed; make the first call
//     on a device before any stream capture;
//   * every call on a device shares the one array and leaves its contents behind: calls whose
//     work overlaps on the GPU (other streams, other threads) race and must be serialised by
//     the caller; nothing in the array needs clearing, the recomputation overwrites every
//     element the backward reads;
//   * du (and dz, with a gate) receive the recomputed forward outputs before the backward
//     overwrites them, so they must not alias any input.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/mamba_b200_ss.h"
#include "ss_common.cuh"  // record_cuda_status, check_bwd

namespace {

static __device__ __align__(256) float g_noalloc_ckpt[SS_NOALLOC_MAX_CKPT_ELEMS];

constexpr int kMaxDevices = 64;

struct ScratchEntry {
  CUcontext ctx;  // context the address was looked up in (null: unknown)
  float* ptr;
};
std::mutex g_setup_mu;
ScratchEntry g_scratch[kMaxDevices] = {};

using CtxGetCurrent = CUresult (*)(CUcontext*);

// cuCtxGetCurrent from the driver, fetched through the runtime (no -lcuda link); null if absent
CtxGetCurrent ctx_get_current() {
  static CtxGetCurrent fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 4000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrent>(p);
    else
      cudaGetLastError();
  });
  return fn;
}

CUcontext current_context() {
  CtxGetCurrent fn = ctx_get_current();
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

// set-up: the device address of g_noalloc_ckpt in the current device's current context (host
// code cannot use the symbol itself — in host code it only names a host-side stand-in)
int scratch_for_current_device(float** out, int* dev_out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return ssb::record_cuda_status(e);
  if (dev < 0 || dev >= kMaxDevices) return SS_ERR_UNSUPPORTED;
  const CUcontext ctx = current_context();
  std::lock_guard<std::mutex> lock(g_setup_mu);
  ScratchEntry& en = g_scratch[dev];
  if (en.ptr == nullptr || ctx == nullptr || en.ctx != ctx) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_ckpt);
    if (e != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      en.ptr = nullptr;
      return ssb::record_cuda_status(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
    }
    en.ptr = static_cast<float*>(p);
    en.ctx = current_context();  // the lookup makes the primary context current if none was
  }
  *out = en.ptr;
  *dev_out = dev;
  return SS_OK;
}

void forget_scratch(int dev) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  g_scratch[dev].ptr = nullptr;
}

}  // namespace

extern "C" SS_API int ss_bwd_noalloc(const ss_bwd_args* args, void* stream) {
  int rc = ssb::check_bwd(args, true);
  if (rc != SS_OK) return rc;
  const ss_fwd_args& f = args->f;
  if (ss_ckpt_elems(f.batch, f.dim, f.seqlen, f.dstate) > (size_t)SS_NOALLOC_MAX_CKPT_ELEMS)
    return SS_ERR_UNSUPPORTED;
  float* scratch = nullptr;
  int dev = -1;
  rc = scratch_for_current_device(&scratch, &dev);
  if (rc != SS_OK) return rc;

  // 1. recompute the states into the scratch array; the forward output lands in du and,
  //    with a gate, the ungated output the backward needs lands in dz
  ss_fwd_args fa = f;
  fa.out = args->du;
  fa.out_batch_stride = args->du_batch_stride;
  fa.out_dim_stride = args->du_dim_stride;
  fa.ckpt = scratch;
  fa.last_state = nullptr;
  fa.out_y = f.z ? args->dz : nullptr;
  fa.out_y_batch_stride = args->dz_batch_stride;
  fa.out_y_dim_stride = args->dz_dim_stride;
  rc = ss_fwd(&fa, stream);

  // 2. the backward from those states (each element of y is read before dz overwrites it)
  if (rc == SS_OK) {
    ss_bwd_args ba = *args;
    ba.f.ckpt = scratch;
    ba.y = fa.out_y;
    ba.y_batch_stride = args->dz_batch_stride;
    ba.y_dim_stride = args->dz_dim_stride;
    rc = ss_bwd(&ba, stream);
  }
  if (rc == SS_ERR_CUDA) forget_scratch(dev);  // look the address up again on the next call
  return rc;
}
