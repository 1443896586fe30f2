// C ABI of the residual-add + RMSNorm kernels: validation and dispatch over dtype and the
// number of 16-byte vectors each lane keeps of a row.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mamba_b200_ss.h"
#include "ss_norm.cuh"

namespace {

using namespace ssb;

bool aligned_rows(const void* p, int64_t stride, size_t es) {
  return p == nullptr || ((reinterpret_cast<uintptr_t>(p) & 15) == 0 && ((stride * (int64_t)es) & 15) == 0);
}

// vectors per lane: the smallest of 1, 2, 3, 4, 6, 8 covering the row (3 fits d_model 768 in
// bf16 exactly); 0 when the row is too long
int vectors_per_lane(int dim, size_t es) {
  const int vw = (int)(16 / es);
  const int need = (dim + 32 * vw - 1) / (32 * vw);
  for (int nv : {1, 2, 3, 4, 6, 8})
    if (need <= nv) return nv;
  return 0;
}

template <typename F>
int by_dtype(int io, F&& f) {
  switch (io) {
    case SS_F32: return record_cuda_status(f(float{}));
    case SS_BF16: return record_cuda_status(f(__nv_bfloat16{}));
    case SS_F16: return record_cuda_status(f(__half{}));
    default: return SS_ERR_UNSUPPORTED;
  }
}

}  // namespace

#define SSB_NORM_LAUNCH(KERNEL)                                                           \
  switch (nv) {                                                                           \
    case 1: KERNEL<IT, 1><<<grid, 32 * kNormWarps, 0, st>>>(P); break;                    \
    case 2: KERNEL<IT, 2><<<grid, 32 * kNormWarps, 0, st>>>(P); break;                    \
    case 3: KERNEL<IT, 3><<<grid, 32 * kNormWarps, 0, st>>>(P); break;                    \
    case 4: KERNEL<IT, 4><<<grid, 32 * kNormWarps, 0, st>>>(P); break;                    \
    case 6: KERNEL<IT, 6><<<grid, 32 * kNormWarps, 0, st>>>(P); break;                    \
    default: KERNEL<IT, 8><<<grid, 32 * kNormWarps, 0, st>>>(P); break;                   \
  }                                                                                       \
  return cudaGetLastError();

extern "C" {

int ss_rmsnorm_fwd(const ss_rmsnorm_args* a, void* stream) {
  if (a == nullptr) return SS_ERR_INVALID;
  if (a->rows < 0 || a->dim < 1 || !(a->eps >= 0.f)) return SS_ERR_INVALID;
  if (a->io_dtype != SS_F32 && a->io_dtype != SS_BF16 && a->io_dtype != SS_F16) return SS_ERR_UNSUPPORTED;
  if (vectors_per_lane(a->dim, a->io_dtype == SS_F32 ? 4 : 2) == 0) return SS_ERR_UNSUPPORTED;
  if (a->rows == 0) return SS_OK;  // empty tensors may carry null data pointers
  if (!a->x || !a->weight || !a->y) return SS_ERR_INVALID;
  if (a->x_row_stride < a->dim || a->y_row_stride < a->dim) return SS_ERR_INVALID;
  if (a->residual && a->residual_row_stride < a->dim) return SS_ERR_INVALID;
  if (a->residual_out && (!a->residual || a->residual_out_row_stride < a->dim)) return SS_ERR_INVALID;
  const size_t es = a->io_dtype == SS_F32 ? 4 : 2;
  const int nv = vectors_per_lane(a->dim, es);
  NormK P;
  P.a = *a;
  P.vec = a->dim % (int)(16 / es) == 0 && aligned_rows(a->x, a->x_row_stride, es) &&
          aligned_rows(a->residual, a->residual_row_stride, es) && aligned_rows(a->y, a->y_row_stride, es) &&
          aligned_rows(a->residual_out, a->residual_out_row_stride, es);
  cudaStream_t st = (cudaStream_t)stream;
  // persistent grid: each warp walks rows with a stride of the grid's warps
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  const int ctas = (a->rows + kNormWarps - 1) / kNormWarps;
  dim3 grid(ctas < 4 * sms ? ctas : 4 * sms);
  return by_dtype(a->io_dtype, [&](auto tag) {
    using IT = decltype(tag);
    SSB_NORM_LAUNCH(rmsnorm_fwd_kernel)
  });
}

int ss_rmsnorm_bwd(const ss_rmsnorm_bwd_args* a, void* stream) {
  if (a == nullptr) return SS_ERR_INVALID;
  if (a->rows < 0 || a->dim < 1) return SS_ERR_INVALID;
  if (a->io_dtype != SS_F32 && a->io_dtype != SS_BF16 && a->io_dtype != SS_F16) return SS_ERR_UNSUPPORTED;
  const size_t es = a->io_dtype == SS_F32 ? 4 : 2;
  const int nv = vectors_per_lane(a->dim, es);
  if (nv == 0) return SS_ERR_UNSUPPORTED;
  if (!a->weight || !a->dweight) return SS_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(a->dweight, 0, sizeof(float) * (size_t)a->dim, st);
  if (e != cudaSuccess) return record_cuda_status(e);
  if (a->rows == 0) return SS_OK;  // empty tensors may carry null data pointers
  if (!a->h || !a->rstd || !a->dy || !a->dh) return SS_ERR_INVALID;
  if (a->h_row_stride < a->dim || a->dy_row_stride < a->dim || a->dh_row_stride < a->dim) return SS_ERR_INVALID;
  if (a->dh_in && a->dh_in_row_stride < a->dim) return SS_ERR_INVALID;
  NormBwdK P;
  P.a = *a;
  P.vec = a->dim % (int)(16 / es) == 0 && aligned_rows(a->h, a->h_row_stride, es) &&
          aligned_rows(a->dy, a->dy_row_stride, es) && aligned_rows(a->dh, a->dh_row_stride, es) &&
          aligned_rows(a->dh_in, a->dh_in_row_stride, es);
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  cudaGetLastError();
  // persistent grid: each warp visits many rows, so dweight costs one atomic per column and CTA
  const int ctas = (a->rows + kNormWarps - 1) / kNormWarps;
  dim3 grid(ctas < 4 * sms ? ctas : 4 * sms);
  return by_dtype(a->io_dtype, [&](auto tag) {
    using IT = decltype(tag);
    SSB_NORM_LAUNCH(rmsnorm_bwd_kernel)
  });
}

}  // extern "C"
