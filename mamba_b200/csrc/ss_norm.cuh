// Residual add + RMSNorm, forward and backward (the reference's RMSNorm, modules/rms_norm.py:
// 21-30, and the residual add of its Block, models/causal_lm.py:30-37):
//
//   h   = x + residual            (rounded to the I/O dtype, as the reference's in-place add)
//   y   = h * rsqrt(mean(h^2) + eps) * (1 + w)      (or * w when unit_offset == 0)
//
// In the reference each of these is a chain of PyTorch kernels (a cast, pow, mean, rsqrt and
// three multiplies for the norm, one add for the residual); here it is one pass per row.
// One warp per row; each lane holds NV 16-byte vectors of the row in registers between the
// statistics and the normalisation, so the row is read once and written once.
//   backward: g = dy * (1 + w); dh = rstd * (g - h * rstd^2 * mean(g h)) (+ the gradient
//   arriving at h); dw = sum over rows of dy * h * rstd, accumulated per lane across the rows a
//   warp visits (persistent grid), reduced per CTA, then one atomic per column and CTA.
#pragma once
#include "ss_common.cuh"

namespace ssb {

constexpr int kNormWarps = 4;

struct NormK {
  ss_rmsnorm_args a;
  int vec;  // all rows 16-byte aligned and dim a multiple of the vector width
};

struct NormBwdK {
  ss_rmsnorm_bwd_args a;
  int vec;
};

// element indices of lane `lane`'s vector j: (j * 32 + lane) * VW + k
template <typename IT, int NV>
__device__ __forceinline__ void row_load(float (&v)[NV][16 / sizeof(IT)], const IT* row, int dim, int lane, bool vec) {
  constexpr int VW = 16 / sizeof(IT);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int e0 = (j * 32 + lane) * VW;
    if (vec && e0 + VW <= dim) {
      const uint4 pk = *reinterpret_cast<const uint4*>(row + e0);
      const IT* e = reinterpret_cast<const IT*>(&pk);
#pragma unroll
      for (int k = 0; k < VW; ++k) v[j][k] = to_f<IT>(e[k]);
    } else {
#pragma unroll
      for (int k = 0; k < VW; ++k) v[j][k] = (e0 + k < dim) ? to_f<IT>(row[e0 + k]) : 0.f;
    }
  }
}

template <typename IT, int NV>
__device__ __forceinline__ void row_store(IT* row, const float (&v)[NV][16 / sizeof(IT)], int dim, int lane,
                                          bool vec) {
  constexpr int VW = 16 / sizeof(IT);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int e0 = (j * 32 + lane) * VW;
    if (vec && e0 + VW <= dim) {
      uint4 pk;
      IT* e = reinterpret_cast<IT*>(&pk);
#pragma unroll
      for (int k = 0; k < VW; ++k) e[k] = from_f<IT>(v[j][k]);
      *reinterpret_cast<uint4*>(row + e0) = pk;
    } else {
#pragma unroll
      for (int k = 0; k < VW; ++k)
        if (e0 + k < dim) row[e0 + k] = from_f<IT>(v[j][k]);
    }
  }
}

template <int NV, int VW>
__device__ __forceinline__ void load_weight(float (&w)[NV][VW], const float* weight, int dim, int lane, bool unit) {
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int k = 0; k < VW; ++k) {
      const int e = (j * 32 + lane) * VW + k;
      w[j][k] = e < dim ? weight[e] + (unit ? 1.f : 0.f) : 0.f;
    }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename IT, int NV>
__global__ void __launch_bounds__(32 * kNormWarps) rmsnorm_fwd_kernel(const __grid_constant__ NormK P) {
  constexpr int VW = 16 / sizeof(IT);
  const ss_rmsnorm_args& a = P.a;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const int dim = a.dim;
  float w[NV][VW];  // issued first: its latency overlaps the row loads
  load_weight<NV, VW>(w, a.weight, dim, lane, a.unit_offset != 0);
  float h[NV][VW];
  row_load<IT, NV>(h, (const IT*)a.x + (int64_t)row * a.x_row_stride, dim, lane, P.vec);
  if (a.residual != nullptr) {
    float r[NV][VW];
    row_load<IT, NV>(r, (const IT*)a.residual + (int64_t)row * a.residual_row_stride, dim, lane, P.vec);
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int k = 0; k < VW; ++k) h[j][k] = to_f<IT>(from_f<IT>(h[j][k] + r[j][k]));  // the I/O-dtype sum
    if (a.residual_out != nullptr)
      row_store<IT, NV>((IT*)a.residual_out + (int64_t)row * a.residual_out_row_stride, h, dim, lane, P.vec);
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int k = 0; k < VW; ++k) ss = fmaf(h[j][k], h[j][k], ss);
  const float rstd = rsqrtf(warp_sum(ss) / (float)dim + a.eps);
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int k = 0; k < VW; ++k) h[j][k] = h[j][k] * rstd * w[j][k];
  row_store<IT, NV>((IT*)a.y + (int64_t)row * a.y_row_stride, h, dim, lane, P.vec);
  if (a.rstd != nullptr && lane == 0) a.rstd[row] = rstd;
}

template <typename IT, int NV>
__global__ void __launch_bounds__(32 * kNormWarps) rmsnorm_bwd_kernel(const __grid_constant__ NormBwdK P) {
  constexpr int VW = 16 / sizeof(IT);
  __shared__ float red[kNormWarps][NV * 32 * VW];
  const ss_rmsnorm_bwd_args& a = P.a;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int dim = a.dim;
  const bool unit = a.unit_offset != 0;
  float dw[NV][VW];  // the weight itself is re-read per row (L1-resident) to keep registers for dw
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int k = 0; k < VW; ++k) dw[j][k] = 0.f;
  const float inv_dim = 1.f / (float)dim;
  for (int row = blockIdx.x * kNormWarps + wid; row < a.rows; row += gridDim.x * kNormWarps) {
    float h[NV][VW], g[NV][VW], gin[NV][VW];
    // all of the row's loads are issued before any is consumed: one memory round trip per row
    row_load<IT, NV>(h, (const IT*)a.h + (int64_t)row * a.h_row_stride, dim, lane, P.vec);
    row_load<IT, NV>(g, (const IT*)a.dy + (int64_t)row * a.dy_row_stride, dim, lane, P.vec);
    if (a.dh_in != nullptr)
      row_load<IT, NV>(gin, (const IT*)a.dh_in + (int64_t)row * a.dh_in_row_stride, dim, lane, P.vec);
    const float rstd = a.rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int k = 0; k < VW; ++k) {
        const int e = (j * 32 + lane) * VW + k;
        const float wk = e < dim ? a.weight[e] + (unit ? 1.f : 0.f) : 0.f;
        dw[j][k] = fmaf(g[j][k], h[j][k] * rstd, dw[j][k]);
        g[j][k] *= wk;
        dot = fmaf(g[j][k], h[j][k], dot);
      }
    const float c = warp_sum(dot) * inv_dim * rstd * rstd;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int k = 0; k < VW; ++k) g[j][k] = rstd * (g[j][k] - h[j][k] * c);
    if (a.dh_in != nullptr) {
#pragma unroll
      for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int k = 0; k < VW; ++k) g[j][k] += gin[j][k];
    }
    row_store<IT, NV>((IT*)a.dh + (int64_t)row * a.dh_row_stride, g, dim, lane, P.vec);
  }
  // dweight: this CTA's warps, then one atomic per column
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int k = 0; k < VW; ++k) red[wid][(j * 32 + lane) * VW + k] = dw[j][k];
  __syncthreads();
  for (int e = threadIdx.x; e < dim && e < NV * 32 * VW; e += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < kNormWarps; ++r) s += red[r][e];
    atomicAdd(a.dweight + e, s);
  }
}

}  // namespace ssb
