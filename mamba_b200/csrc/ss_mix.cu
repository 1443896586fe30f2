// C ABI of the fused decode mixer step (ss_mamba_step): validation, cluster size and dispatch.
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/mamba_b200_ss.h"
#include "ss_mix.cuh"

namespace {

using namespace ssb;

template <typename IT, int K, int TPC, int R, int CL>
cudaError_t launch_mix(const MixK& P, cudaStream_t st) {
  const size_t smem = sizeof(float) * ((size_t)P.cs + 2 * (size_t)P.J);
  auto kern = mamba_step_kernel<IT, K, TPC, R, CL>;
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  kern<<<dim3((unsigned)((int64_t)P.a.batch * CL)), kMixThreads, smem, st>>>(P);
  return cudaGetLastError();
}

template <typename IT, int K, int TPC, int R>
cudaError_t by_cluster(int cl, const MixK& P, cudaStream_t st) {
  switch (cl) {
    case 1: return launch_mix<IT, K, TPC, R, 1>(P, st);
    case 2: return launch_mix<IT, K, TPC, R, 2>(P, st);
    case 4: return launch_mix<IT, K, TPC, R, 4>(P, st);
    default: return launch_mix<IT, K, TPC, R, 8>(P, st);
  }
}

// lanes per channel in the SSM phase: 1, 2, 4 for dstate <= 4, 8, 16; 32 lanes with one or
// two 128-state chunks above
template <typename IT, int K>
cudaError_t by_tpc(int dstate, int cl, const MixK& P, cudaStream_t st) {
  if (dstate <= 4) return by_cluster<IT, K, 1, 1>(cl, P, st);
  if (dstate <= 8) return by_cluster<IT, K, 2, 1>(cl, P, st);
  if (dstate <= 16) return by_cluster<IT, K, 4, 1>(cl, P, st);
  if (dstate <= 128) return by_cluster<IT, K, 32, 1>(cl, P, st);
  return by_cluster<IT, K, 32, 2>(cl, P, st);
}

template <typename IT>
cudaError_t by_width(int K, int dstate, int cl, const MixK& P, cudaStream_t st) {
  switch (K) {
    case 1: return by_tpc<IT, 1>(dstate, cl, P, st);
    case 2: return by_tpc<IT, 2>(dstate, cl, P, st);
    case 3: return by_tpc<IT, 3>(dstate, cl, P, st);
    default: return by_tpc<IT, 4>(dstate, cl, P, st);
  }
}

}  // namespace

extern "C" {

int ss_mamba_step(const ss_mamba_step_args* a, void* stream) {
  if (a == nullptr) return SS_ERR_INVALID;
  if (a->batch < 0 || a->dim < 1 || a->dstate < 1 || a->width < 1 || a->dt_rank < 1) return SS_ERR_INVALID;
  if (a->dstate > SS_MAX_DSTATE || a->width > SS_MAX_CONV_WIDTH || (int64_t)a->batch * 8 > 2147483647LL)
    return SS_ERR_UNSUPPORTED;
  if (a->io_dtype != SS_F32 && a->io_dtype != SS_BF16 && a->io_dtype != SS_F16) return SS_ERR_UNSUPPORTED;
  const int J = a->dt_rank + 2 * a->dstate;
  if (J > 4096) return SS_ERR_UNSUPPORTED;
  if (!a->conv_weight || !a->x_proj || !a->dt_proj || !a->A) return SS_ERR_INVALID;
  if (a->xz_batch_stride < 2LL * a->dim || a->y_batch_stride < a->dim) return SS_ERR_INVALID;
  if (a->batch == 0) return SS_OK;  // the per-sequence tensors are empty and may carry null pointers
  if (!a->xz || !a->ssm_state || !a->y || (a->width > 1 && !a->conv_state)) return SS_ERR_INVALID;
  // a cluster of cl CTAs per sequence, so that batch x cl covers about two CTAs per SM, each
  // CTA keeping at least 32 channels
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  int cl = 1;
  while (cl < 8 && a->batch * cl < 2 * sms && (a->dim + 2 * cl - 1) / (2 * cl) >= 32) cl *= 2;
  MixK P{};  // every field is set below; value-initialised so none is ever read uninitialised
  P.a = *a;
  P.J = J;
  P.cs = (((a->dim + cl - 1) / cl) + 31) / 32 * 32;
  const size_t es = a->io_dtype == SS_F32 ? 4 : 2;
  P.vec_x = (reinterpret_cast<uintptr_t>(a->x_proj) & 15) == 0 && ((a->dim * es) & 15) == 0;
  P.vec_a = a->dstate % 4 == 0 && (reinterpret_cast<uintptr_t>(a->A) & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(a->ssm_state) & 15) == 0;
  if (sizeof(float) * ((size_t)P.cs + 2 * (size_t)J) > 200 * 1024) return SS_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  switch (a->io_dtype) {
    case SS_F32: return record_cuda_status(by_width<float>(a->width, a->dstate, cl, P, st));
    case SS_BF16: return record_cuda_status(by_width<__nv_bfloat16>(a->width, a->dstate, cl, P, st));
    default: return record_cuda_status(by_width<__half>(a->width, a->dstate, cl, P, st));
  }
}

}  // extern "C"
