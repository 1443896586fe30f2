// C ABI of the input-side convolution (ss_conv_fwd / ss_conv_bwd / ss_conv_step):
// validation, vector-path flags and dispatch over dtype, width and the z copy.
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

#include "../../include/mamba_b200_ss.h"
#include "ss_conv.cuh"

namespace {

using namespace ssb;

size_t es_of(int dt) { return dt == SS_F32 ? 4 : 2; }
bool dt_ok(int dt) { return dt == SS_F32 || dt == SS_BF16 || dt == SS_F16; }

// rows of a (batch, outer, inner) view with unit inner stride start 16-byte aligned
bool al16(const void* p, int64_t s0, int64_t s1, size_t es) {
  return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && ((s0 * (int64_t)es) & 15) == 0 &&
         ((s1 * (int64_t)es) & 15) == 0;
}

int check_conv(const ss_conv_args* a) {
  if (a == nullptr) return SS_ERR_INVALID;
  if (a->batch < 0 || a->dim < 1 || a->seqlen < 0 || a->width < 1) return SS_ERR_INVALID;
  if (a->width > SS_MAX_CONV_WIDTH) return SS_ERR_UNSUPPORTED;
  if ((int64_t)a->batch * (((int64_t)a->seqlen + kConvT - 1) / kConvT) * ((a->dim + kConvC - 1) / kConvC) >
      2147483647LL)
    return SS_ERR_UNSUPPORTED;
  if (!dt_ok(a->io_dtype)) return SS_ERR_UNSUPPORTED;
  // empty tensors (no batch rows or no steps) may carry null data pointers
  if (!a->weight || (!a->x && a->batch > 0 && a->seqlen > 0)) return SS_ERR_INVALID;
  if (a->x_batch_stride < 0 || a->x_seq_stride < 0) return SS_ERR_INVALID;
  if (a->state_out != nullptr && a->state_out == a->state_in) return SS_ERR_INVALID;
  return SS_OK;
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

template <typename F>
cudaError_t by_width(int w, F&& f) {
  switch (w) {
    case 1: return f(std::integral_constant<int, 1>{});
    case 2: return f(std::integral_constant<int, 2>{});
    case 3: return f(std::integral_constant<int, 3>{});
    default: return f(std::integral_constant<int, 4>{});
  }
}

}  // namespace

extern "C" {

int ss_conv_fwd(const ss_conv_args* a, void* stream) {
  int s = check_conv(a);
  if (s != SS_OK) return s;
  if ((!a->u && a->batch > 0 && a->seqlen > 0) || a->u_batch_stride < 0 || a->u_dim_stride < 0) return SS_ERR_INVALID;
  if (a->z && (!a->zt || a->z_batch_stride < 0 || a->z_seq_stride < 0 || a->zt_batch_stride < 0 ||
               a->zt_dim_stride < 0))
    return SS_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  const int K = a->width;
  if (a->batch == 0) return SS_OK;
  if (a->seqlen == 0) {  // nothing to convolve; the state passes through unchanged
    if (a->state_out == nullptr || K == 1) return SS_OK;
    const size_t bytes = (size_t)a->batch * a->dim * (K - 1) * sizeof(float);
    return record_cuda_status(a->state_in ? cudaMemcpyAsync(a->state_out, a->state_in, bytes,
                                                            cudaMemcpyDeviceToDevice, st)
                                          : cudaMemsetAsync(a->state_out, 0, bytes, st));
  }
  const size_t es = es_of(a->io_dtype);
  const int vw = (int)(16 / es);
  ConvK P;
  P.a = *a;
  P.vec_x = al16(a->x, a->x_batch_stride, a->x_seq_stride, es) && a->dim % vw == 0;
  P.vec_u = al16(a->u, a->u_batch_stride, a->u_dim_stride, es);
  P.vec_z = a->z ? (al16(a->z, a->z_batch_stride, a->z_seq_stride, es) && a->dim % vw == 0) : 0;
  P.vec_zt = a->z ? al16(a->zt, a->zt_batch_stride, a->zt_dim_stride, es) : 0;
  P.nc = (a->dim + kConvC - 1) / kConvC;
  P.nt = (a->seqlen + kConvT - 1) / kConvT;
  dim3 grid((unsigned)((int64_t)a->batch * P.nt * P.nc));
  return by_dtype(a->io_dtype, [&](auto tag) {
    using IT = decltype(tag);
    return by_width(K, [&](auto kc) {
      constexpr int KK = decltype(kc)::value;
      const size_t smem = sizeof(ConvFwdSmem<IT, KK>);
      auto kern = a->z ? conv_fwd_kernel<IT, KK, true> : conv_fwd_kernel<IT, KK, false>;
      cudaError_t e2 = ensure_smem_limit(reinterpret_cast<const void*>(kern), smem);
      if (e2 != cudaSuccess) return e2;
      kern<<<grid, kConvThreads, smem, st>>>(P);
      return cudaGetLastError();
    });
  });
}

int ss_conv_bwd(const ss_conv_bwd_args* a, void* stream) {
  if (a == nullptr) return SS_ERR_INVALID;
  int s = check_conv(&a->f);
  if (s != SS_OK) return s;
  if (!a->dweight || ((!a->du || !a->dx) && a->f.batch > 0 && a->f.seqlen > 0)) return SS_ERR_INVALID;
  if (a->du_batch_stride < 0 || a->du_dim_stride < 0 || a->dx_batch_stride < 0 || a->dx_seq_stride < 0)
    return SS_ERR_INVALID;
  if (a->dzt && (!a->dz || a->dzt_batch_stride < 0 || a->dzt_dim_stride < 0 || a->dz_batch_stride < 0 ||
                 a->dz_seq_stride < 0))
    return SS_ERR_INVALID;
  const ss_conv_args& f = a->f;
  cudaStream_t st = (cudaStream_t)stream;
  const int K = f.width;
  cudaError_t e = cudaMemsetAsync(a->dweight, 0, sizeof(float) * (size_t)f.dim * K, st);
  if (e == cudaSuccess && a->dbias) e = cudaMemsetAsync(a->dbias, 0, sizeof(float) * (size_t)f.dim, st);
  if (e != cudaSuccess) return record_cuda_status(e);
  if (f.batch == 0 || f.seqlen == 0) return SS_OK;
  const size_t es = es_of(f.io_dtype);
  const int vw = (int)(16 / es);
  ConvBwdK P;
  P.a = *a;
  P.vec_x = al16(f.x, f.x_batch_stride, f.x_seq_stride, es) && f.dim % vw == 0;
  P.vec_du = al16(a->du, a->du_batch_stride, a->du_dim_stride, es);
  P.vec_dx = al16(a->dx, a->dx_batch_stride, a->dx_seq_stride, es) && f.dim % vw == 0;
  P.vec_dzt = a->dzt ? al16(a->dzt, a->dzt_batch_stride, a->dzt_dim_stride, es) : 0;
  P.vec_dz = a->dzt ? (al16(a->dz, a->dz_batch_stride, a->dz_seq_stride, es) && f.dim % vw == 0) : 0;
  P.nc = (f.dim + kConvC - 1) / kConvC;
  P.nt = (f.seqlen + kConvT - 1) / kConvT;
  dim3 grid((unsigned)((int64_t)f.batch * P.nt * P.nc));
  return by_dtype(f.io_dtype, [&](auto tag) {
    using IT = decltype(tag);
    return by_width(K, [&](auto kc) {
      constexpr int KK = decltype(kc)::value;
      const size_t smem = sizeof(ConvBwdSmem<IT, KK>);
      auto kern = a->dzt ? conv_bwd_kernel<IT, KK, true> : conv_bwd_kernel<IT, KK, false>;
      cudaError_t e2 = ensure_smem_limit(reinterpret_cast<const void*>(kern), smem);
      if (e2 != cudaSuccess) return e2;
      kern<<<grid, kConvThreads, smem, st>>>(P);
      return cudaGetLastError();
    });
  });
}

int ss_conv_step(const ss_conv_step_args* a, void* stream) {
  if (a == nullptr) return SS_ERR_INVALID;
  if (a->batch < 0 || a->dim < 1 || a->width < 1) return SS_ERR_INVALID;
  if (a->width > SS_MAX_CONV_WIDTH) return SS_ERR_UNSUPPORTED;
  const int ncb = (a->dim + 127) / 128;
  if ((int64_t)a->batch * ncb > 2147483647LL) return SS_ERR_UNSUPPORTED;
  if (!dt_ok(a->io_dtype)) return SS_ERR_UNSUPPORTED;
  if (!a->weight || a->state_batch_stride < 0 || a->x_batch_stride < 0 || a->u_batch_stride < 0)
    return SS_ERR_INVALID;
  if (a->batch == 0) return SS_OK;  // empty tensors may carry null data pointers
  if (!a->x || !a->u || (a->width > 1 && !a->state)) return SS_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid((unsigned)((int64_t)a->batch * ncb));
  return by_dtype(a->io_dtype, [&](auto tag) {
    using IT = decltype(tag);
    return by_width(a->width, [&](auto kc) {
      conv_step_kernel<IT, decltype(kc)::value><<<grid, 128, 0, st>>>(*a, ncb);
      return cudaGetLastError();
    });
  });
}

}  // extern "C"
