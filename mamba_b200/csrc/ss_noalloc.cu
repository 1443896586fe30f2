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
//   * the first call on a device looks up the scratch array's device address (set-up, once
//     per device, with that device current); make that first call before any stream capture;
//   * every call on a device shares the one array and leaves its contents behind: calls whose
//     work overlaps on the GPU (other streams, other threads) race and must be serialised by
//     the caller; nothing in the array needs clearing, the recomputation overwrites every
//     element the backward reads;
//   * du (and dz, with a gate) receive the recomputed forward outputs before the backward
//     overwrites them, so they must not alias any input.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/mamba_b200_ss.h"

namespace {

static __device__ __align__(256) float g_noalloc_ckpt[SS_NOALLOC_MAX_CKPT_ELEMS];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
float* g_scratch[kMaxDevices] = {};

// set-up: the device address of g_noalloc_ckpt on the current device (host code cannot use
// the symbol itself — in host code it only names a host-side stand-in)
int scratch_for_current_device(float** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SS_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_ckpt) != cudaSuccess || p == nullptr) {
      cudaGetLastError();
      return SS_ERR_CUDA;
    }
    g_scratch[dev] = static_cast<float*>(p);
  }
  *out = g_scratch[dev];
  return SS_OK;
}

}  // namespace

extern "C" SS_API int ss_bwd_noalloc(const ss_bwd_args* args, void* stream) {
  if (args == nullptr) return SS_ERR_INVALID;
  const ss_fwd_args& f = args->f;
  if (f.batch < 0 || f.dim < 1 || f.seqlen < 0 || f.dstate < 1) return SS_ERR_INVALID;
  if (ss_ckpt_elems(f.batch, f.dim, f.seqlen, f.dstate) > (size_t)SS_NOALLOC_MAX_CKPT_ELEMS)
    return SS_ERR_UNSUPPORTED;
  if (args->du == nullptr && f.batch > 0 && f.seqlen > 0) return SS_ERR_INVALID;  // empty: may be null
  float* scratch = nullptr;
  int rc = scratch_for_current_device(&scratch);
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
  if (rc != SS_OK) return rc;

  // 2. the backward from those states (each element of y is read before dz overwrites it)
  ss_bwd_args ba = *args;
  ba.f.ckpt = scratch;
  ba.y = fa.out_y;
  ba.y_batch_stride = args->dz_batch_stride;
  ba.y_dim_stride = args->dz_dim_stride;
  return ss_bwd(&ba, stream);
}
