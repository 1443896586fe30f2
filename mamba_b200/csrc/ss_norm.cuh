// Residual add + RMSNorm, forward and backward (the reference's RMSNorm, modules/rms_norm.py:
// 21-30, and the residual add of its Block, models/causal_lm.py:30-37):
//
//   h   = x + residual            (rounded to the I/O dtype, as the reference's in-place add)
//   y   = h * rsqrt(mean(h^2) + eps) * (1 + w)      (or * w when unit_offset == 0)
//
// In the reference each of these is a chain of PyTorch kernels (a cast, pow, mean, rsqrt and
// three multiplies for the norm, one add for the residual); here it is one pass per row.
// One warp per row at a time, persistent over rows; each lane holds NV 16-byte vectors of the
// row in registers between the statistics and the normalisation, so the row is read once and
// written once, and the next row's loads are already in flight while a row is computed.
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

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// lane `lane`'s NV vectors of a row kept packed in the I/O dtype (16 bytes each): half the
// registers of the unpacked row, so a warp can hold the next row's loads while it works
template <typename IT, int NV>
__device__ __forceinline__ void row_load_packed(uint4 (&q)[NV], const IT* row, int dim, int lane, bool vec) {
  constexpr int VW = 16 / sizeof(IT);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int e0 = (j * 32 + lane) * VW;
    if (vec && e0 + VW <= dim) {
      q[j] = *reinterpret_cast<const uint4*>(row + e0);
    } else {
      union { uint4 u; IT e[VW]; } pk;
#pragma unroll
      for (int k = 0; k < VW; ++k) pk.e[k] = (e0 + k < dim) ? row[e0 + k] : zero_v<IT>();
      q[j] = pk.u;
    }
  }
}

template <typename IT, int NV>
__device__ __forceinline__ void unpack_row(float (&v)[NV][16 / sizeof(IT)], const uint4 (&q)[NV]) {
  constexpr int VW = 16 / sizeof(IT);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const IT* e = reinterpret_cast<const IT*>(&q[j]);
#pragma unroll
    for (int k = 0; k < VW; ++k) v[j][k] = to_f<IT>(e[k]);
  }
}

// (1 + weight) or weight for the CTA's rows, in shared memory
template <int LEN>
__device__ __forceinline__ void fill_weight(float* w_s, const float* weight, int dim, bool unit) {
  const float ofs = unit ? 1.f : 0.f;
  for (int e = threadIdx.x; e < LEN; e += blockDim.x) w_s[e] = e < dim ? weight[e] + ofs : 0.f;
}

// Persistent warps: warp i handles rows i, i + W, i + 2W, ... (W warps in the grid); the next
// row's x / residual loads are issued before the current row is used, so two rows per warp
// are in flight.  The first row's loads go out before the weight is staged.
template <typename IT, int NV>
__global__ void __launch_bounds__(32 * kNormWarps) rmsnorm_fwd_kernel(const __grid_constant__ NormK P) {
  constexpr int VW = 16 / sizeof(IT);
  constexpr int LEN = NV * 32 * VW;
  constexpr bool kLook = NV <= 4;  // wider rows would spill the lookahead registers
  __shared__ __align__(16) float w_s[LEN];
  const ss_rmsnorm_args& a = P.a;
  const int lane = threadIdx.x & 31;
  const int dim = a.dim;
  const bool has_res = a.residual != nullptr;
  const int stride = gridDim.x * kNormWarps;
  int row = blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  uint4 xq[NV], rq[NV];
  if (kLook && row < a.rows) {
    row_load_packed<IT, NV>(xq, (const IT*)a.x + (int64_t)row * a.x_row_stride, dim, lane, P.vec);
    if (has_res) row_load_packed<IT, NV>(rq, (const IT*)a.residual + (int64_t)row * a.residual_row_stride, dim, lane, P.vec);
  }
  fill_weight<LEN>(w_s, a.weight, dim, a.unit_offset != 0);
  __syncthreads();
  for (; row < a.rows; row += stride) {
    if constexpr (!kLook) {
      row_load_packed<IT, NV>(xq, (const IT*)a.x + (int64_t)row * a.x_row_stride, dim, lane, P.vec);
      if (has_res) row_load_packed<IT, NV>(rq, (const IT*)a.residual + (int64_t)row * a.residual_row_stride, dim, lane, P.vec);
    }
    const int next = row + stride;
    uint4 xn[NV], rn[NV];
    if (kLook && next < a.rows) {
      row_load_packed<IT, NV>(xn, (const IT*)a.x + (int64_t)next * a.x_row_stride, dim, lane, P.vec);
      if (has_res) row_load_packed<IT, NV>(rn, (const IT*)a.residual + (int64_t)next * a.residual_row_stride, dim, lane, P.vec);
    }
    float h[NV][VW];
    unpack_row<IT, NV>(h, xq);
    if (has_res) {
      float r[NV][VW];
      unpack_row<IT, NV>(r, rq);
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
      for (int k = 0; k < VW; ++k) h[j][k] = h[j][k] * rstd * w_s[(j * 32 + lane) * VW + k];
    row_store<IT, NV>((IT*)a.y + (int64_t)row * a.y_row_stride, h, dim, lane, P.vec);
    if (a.rstd != nullptr && lane == 0) a.rstd[row] = rstd;
    if (kLook && next < a.rows) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        xq[j] = xn[j];
        if (has_res) rq[j] = rn[j];
      }
    }
  }
}

// Persistent warps as in the forward; the next row's h / dy loads (and its rstd) are issued
// before the current row is used; dh_in, needed last, is loaded at the start of its own row.
template <typename IT, int NV>
__global__ void __launch_bounds__(32 * kNormWarps) rmsnorm_bwd_kernel(const __grid_constant__ NormBwdK P) {
  constexpr int VW = 16 / sizeof(IT);
  constexpr int LEN = NV * 32 * VW;
  constexpr bool kLook = NV <= 3;  // wider rows would spill the lookahead registers
  __shared__ __align__(16) float w_s[LEN];
  __shared__ float red[kNormWarps][LEN];
  const ss_rmsnorm_bwd_args& a = P.a;
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  const int dim = a.dim;
  const int stride = gridDim.x * kNormWarps;
  float dw[NV][VW];
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int k = 0; k < VW; ++k) dw[j][k] = 0.f;
  const float inv_dim = 1.f / (float)dim;
  int row = blockIdx.x * kNormWarps + wid;
  uint4 hq[NV], gq[NV];
  float rstd_c = 0.f;
  if (kLook && row < a.rows) {
    row_load_packed<IT, NV>(hq, (const IT*)a.h + (int64_t)row * a.h_row_stride, dim, lane, P.vec);
    row_load_packed<IT, NV>(gq, (const IT*)a.dy + (int64_t)row * a.dy_row_stride, dim, lane, P.vec);
    rstd_c = a.rstd[row];
  }
  fill_weight<LEN>(w_s, a.weight, dim, a.unit_offset != 0);
  __syncthreads();
  for (; row < a.rows; row += stride) {
    if constexpr (!kLook) {
      row_load_packed<IT, NV>(hq, (const IT*)a.h + (int64_t)row * a.h_row_stride, dim, lane, P.vec);
      row_load_packed<IT, NV>(gq, (const IT*)a.dy + (int64_t)row * a.dy_row_stride, dim, lane, P.vec);
      rstd_c = a.rstd[row];
    }
    uint4 iq[NV];
    if (a.dh_in != nullptr)
      row_load_packed<IT, NV>(iq, (const IT*)a.dh_in + (int64_t)row * a.dh_in_row_stride, dim, lane, P.vec);
    const int next = row + stride;
    uint4 hn[NV], gn[NV];
    float rstd_n = 0.f;
    if (kLook && next < a.rows) {
      row_load_packed<IT, NV>(hn, (const IT*)a.h + (int64_t)next * a.h_row_stride, dim, lane, P.vec);
      row_load_packed<IT, NV>(gn, (const IT*)a.dy + (int64_t)next * a.dy_row_stride, dim, lane, P.vec);
      rstd_n = a.rstd[next];
    }
    const float rstd = rstd_c;
    float h[NV][VW], g[NV][VW];
    unpack_row<IT, NV>(h, hq);
    unpack_row<IT, NV>(g, gq);
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
      for (int k = 0; k < VW; ++k) {
        const float wk = w_s[(j * 32 + lane) * VW + k];
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
      float gi[NV][VW];
      unpack_row<IT, NV>(gi, iq);
#pragma unroll
      for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int k = 0; k < VW; ++k) g[j][k] += gi[j][k];
    }
    row_store<IT, NV>((IT*)a.dh + (int64_t)row * a.dh_row_stride, g, dim, lane, P.vec);
    if (kLook && next < a.rows) {
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        hq[j] = hn[j];
        gq[j] = gn[j];
      }
      rstd_c = rstd_n;
    }
  }
  // dweight: this CTA's warps, then one atomic per column
#pragma unroll
  for (int j = 0; j < NV; ++j)
#pragma unroll
    for (int k = 0; k < VW; ++k) red[wid][(j * 32 + lane) * VW + k] = dw[j][k];
  __syncthreads();
  for (int e = threadIdx.x; e < dim && e < LEN; e += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < kNormWarps; ++r) s += red[r][e];
    atomicAdd(a.dweight + e, s);
  }
}

}  // namespace ssb
