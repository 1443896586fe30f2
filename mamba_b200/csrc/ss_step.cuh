// Single-token decode step (no counterpart in the reference, whose generate() is a stub,
// models/causal_lm.py:61-62): one step of the forward recurrence from a stored state,
//   dt'      = softplus(dt + dt_bias)   (threshold 20, as forward_kernel.cu:216-221), where dt
//              is optionally the delta projection dt_in . dt_proj[c, :] computed here
//   state[n] = exp(dt' A[c,n]) state[n] + dt' x B[n]
//   out      = (sum_n C[n] state[n] + D x) [* silu(z)]
// Bandwidth-bound on the fp32 state (read + write 8 B per (b, c, n)).  TPC threads per
// channel, each holding 4 consecutive states per chunk (one 16-byte access) for R chunks
// (state n = 4 (q + TPC r) + j for lane q of the channel), keep every state access coalesced;
// the output sum over states is a shuffle over the TPC adjacent lanes.  TPC = 1, 2, 4 covers
// dstate <= 16; 8, 16, 32 (with R = 2 above 128) the reference's range up to 256.  The grid is
// flattened over (batch row, channel block), so batch is not bound by gridDim.y.
#pragma once
#include "ss_common.cuh"

namespace ssb {

template <typename IT, int TPC, int R>
__global__ void __launch_bounds__(128) ss_step_kernel(const __grid_constant__ ss_step_args a, int nblk) {
  constexpr int CPB = 128 / TPC;  // channels per block
  const int tid = threadIdx.x;
  const int q = tid % TPC;
  const int c = (blockIdx.x % nblk) * CPB + tid / TPC;
  const int b = blockIdx.x / nblk;
  const int N = a.dstate;
  const bool ok = c < a.dim;
  const int cc = ok ? c : 0;
  const int g = cc / (a.dim / a.ngroups);
  const bool bc_f32 = a.bc_dtype == SS_F32;

  float xv = 0.f, dv = 0.f, zv = 0.f;
  float* st = a.state + (int64_t)b * a.state_batch_stride + (int64_t)cc * N;
  // issue the state loads before the dt work, so their DRAM latency overlaps it
  const bool vec = (N % 4) == 0 && ((reinterpret_cast<uintptr_t>(st) & 15) == 0);
  float s[R][kSPW];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int nb = 4 * (q + TPC * r);
    if (ok && vec && nb < N) {
      const float4 v = *reinterpret_cast<const float4*>(st + nb);
      s[r][0] = v.x; s[r][1] = v.y; s[r][2] = v.z; s[r][3] = v.w;
    } else {
#pragma unroll
      for (int j = 0; j < kSPW; ++j) s[r][j] = (ok && nb + j < N) ? st[nb + j] : 0.f;
    }
  }
  if (a.dt_proj != nullptr) {
    // fused delta projection: the channel's TPC lanes split the dt_rank-long dot product,
    // two independent accumulators per lane
    const IT* din = (const IT*)a.dt + (int64_t)b * a.dt_batch_stride;
    const IT* wrow = (const IT*)a.dt_proj + (int64_t)cc * a.dt_rank;
    float d1 = 0.f;
    int r = q;
#pragma unroll 4
    for (; r + TPC < a.dt_rank; r += 2 * TPC) {
      dv = fmaf(to_f<IT>(din[r]), to_f<IT>(wrow[r]), dv);
      d1 = fmaf(to_f<IT>(din[r + TPC]), to_f<IT>(wrow[r + TPC]), d1);
    }
    if (r < a.dt_rank) dv = fmaf(to_f<IT>(din[r]), to_f<IT>(wrow[r]), dv);
    dv += d1;
#pragma unroll
    for (int o = 1; o < TPC; o <<= 1) dv += __shfl_xor_sync(0xffffffffu, dv, o);
  }
  if (ok) {
    xv = to_f<IT>(((const IT*)a.x)[(int64_t)b * a.x_batch_stride + c]);
    if (a.dt_proj == nullptr) dv = to_f<IT>(((const IT*)a.dt)[(int64_t)b * a.dt_batch_stride + c]);
    if (a.dt_bias != nullptr) dv += a.dt_bias[c];
    if (a.z != nullptr) zv = to_f<IT>(((const IT*)a.z)[(int64_t)b * a.z_batch_stride + c]);
  }
  const float dt = a.dt_softplus ? softplus_thr(dv) : dv;
  const int64_t bsb = a.B_batch_stride ? a.B_batch_stride : (int64_t)a.ngroups * N;
  const int64_t bsc = a.C_batch_stride ? a.C_batch_stride : (int64_t)a.ngroups * N;
  const int64_t bob = (int64_t)b * bsb + (int64_t)g * N, boc = (int64_t)b * bsc + (int64_t)g * N;

  float y = 0.f;
  if (ok) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int nb = 4 * (q + TPC * r);
#pragma unroll
      for (int j = 0; j < kSPW; ++j) {
        const int n = nb + j;
        if (n < N) {
          const float Bn = bc_f32 ? ((const float*)a.B)[bob + n] : to_f<IT>(((const IT*)a.B)[bob + n]);
          const float Cn = bc_f32 ? ((const float*)a.C)[boc + n] : to_f<IT>(((const IT*)a.C)[boc + n]);
          s[r][j] = fmaf(exp_fast(dt * a.A[(int64_t)c * N + n]), s[r][j], dt * xv * Bn);
          y = fmaf(Cn, s[r][j], y);
        }
      }
      if (vec && nb < N) {
        *reinterpret_cast<float4*>(st + nb) = make_float4(s[r][0], s[r][1], s[r][2], s[r][3]);
      } else {
#pragma unroll
        for (int j = 0; j < kSPW; ++j)
          if (nb + j < N) st[nb + j] = s[r][j];
      }
    }
  }
#pragma unroll
  for (int o = 1; o < TPC; o <<= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
  if (ok && q == 0) {
    if (a.D != nullptr) y = fmaf(a.D[c], xv, y);
    if (a.z != nullptr) y *= zv * sigmoid_fast(zv);
    ((IT*)a.out)[(int64_t)b * a.out_batch_stride + c] = from_f<IT>(y);
  }
}

// Lanes per channel and 4-state chunks per lane for a dstate (<= SS_MAX_DSTATE).
inline void step_shape(int dstate, int& tpc, int& chunks) {
  const int quads = (dstate + 3) / 4;
  tpc = 1;
  while (tpc < quads && tpc < 32) tpc *= 2;
  chunks = (quads + tpc - 1) / tpc;
}

}  // namespace ssb
