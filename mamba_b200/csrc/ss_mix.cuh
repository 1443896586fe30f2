// One decode step of a Mamba block's mixer — everything between the input projection and
// the output projection — in one kernel:
//
//   x, z   = the two halves of xz[b]                      (modules/mamba_simple.py:93-97)
//   u      = silu(conv_bias + conv_w . [conv_state, x])   (:97-98; the state then rolls)
//   dbl    = x_proj . u  -> dt_in (dt_rank), B (N), C (N)  (:100-111)
//   dt     = softplus(dt_proj . dt_in + dt_bias)          (:114, forward_kernel.cu:216-221)
//   state  = exp(dt A) state + dt u B;  y = (C . state + D u) * silu(z)
//
// which otherwise takes a conv-step kernel, an x-projection GEMM and the SSM-step kernel.
// A thread-block cluster of CL CTAs serves one sequence (batch row); CTA r owns channels
// [r * cs, (r + 1) * cs): it runs their conv step (so each conv-state entry has one owner),
// forms its partial x projection over them, and the CL partial vectors (dt_rank + 2N floats each)
// are summed through distributed shared memory between two cluster barriers that every
// thread reaches (no early exit).  Each CTA then updates the SSM state of its channels.
// The x projection reads its weight rows once per CTA (from L2); the state traffic is the
// same as the separate SSM-step kernel's.
#pragma once
#include <cooperative_groups.h>

#include "ss_common.cuh"

namespace ssb {

constexpr int kMixThreads = 256;

struct MixK {
  ss_mamba_step_args a;
  int cs;     // channels per CTA (a multiple of 32)
  int J;      // dt_rank + 2 dstate
  int vec_x;  // x_proj rows start 16-byte aligned
  int vec_a;  // A and the SSM state 16-byte aligned with dstate % 4 == 0
};

__device__ __forceinline__ float mix_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// TPC lanes per channel in the SSM phase, each holding R chunks of 4 states (state
// n = 4 (q + TPC r) + j): TPC = 1, 2, 4 for dstate <= 16, TPC = 32 with R = 1 or 2 above.
template <typename IT, int K, int TPC, int R, int CL>
__global__ void __cluster_dims__(CL, 1, 1) __launch_bounds__(kMixThreads)
    mamba_step_kernel(const __grid_constant__ MixK P) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
  const ss_mamba_step_args& a = P.a;
  const int rank = (int)cluster.block_rank();
  const int b = blockIdx.x / CL;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int d = a.dim, N = a.dstate, J = P.J, cs = P.cs;
  const int c_begin = rank * cs, c_end = min(d, c_begin + cs);
  extern __shared__ __align__(16) float mix_smem[];
  float* u_s = mix_smem;       // [cs]  this CTA's u (rounded to the I/O dtype, as a stored activation)
  float* part = u_s + cs;      // [J]   partial x projection over this CTA's channels
  float* dbl = part + J;       // [J]   the full x projection (rounded to the I/O dtype)
  const IT* xb = (const IT*)a.xz + (int64_t)b * a.xz_batch_stride;

  // 1. conv step of this CTA's channels; the conv state rolls in place
  for (int c = c_begin + tid; c < c_end; c += kMixThreads) {
    float* st = a.conv_state + ((int64_t)b * d + c) * (K - 1);
    float win[K];
#pragma unroll
    for (int k = 0; k < K - 1; ++k) win[k] = st[k];
    win[K - 1] = to_f<IT>(xb[c]);
    float p = a.conv_bias != nullptr ? a.conv_bias[c] : 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) p = fmaf(a.conv_weight[(int64_t)c * K + k], win[k], p);
    u_s[c - c_begin] = to_f<IT>(from_f<IT>(p * sigmoid_fast(p)));
#pragma unroll
    for (int k = 0; k < K - 1; ++k) st[k] = win[k + 1];
  }
  __syncthreads();

  // 2. partial x projection over this CTA's channels: each warp takes 4 output rows at a time,
  //    each lane 16-byte vectors of channels, so a lane has several independent weight loads
  //    in flight instead of one dependent chain per row
  {
    constexpr int VW = 16 / sizeof(IT);
    const int len = c_end - c_begin;
    const int nvec = len / VW;  // whole vectors (cs is a multiple of 32; a short last slice has a tail)
    const bool vec_ok = P.vec_x != 0;
    for (int j0 = wid * 4; j0 < J; j0 += (kMixThreads / 32) * 4) {
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      const IT* wr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) wr[i] = (const IT*)a.x_proj + (int64_t)min(j0 + i, J - 1) * d + c_begin;
      if (vec_ok) {
        for (int v = lane; v < nvec; v += 32) {
          uint4 wq[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) wq[i] = *reinterpret_cast<const uint4*>(wr[i] + v * VW);
          float uv[VW];
#pragma unroll
          for (int k = 0; k < VW; ++k) uv[k] = u_s[v * VW + k];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const IT* e = reinterpret_cast<const IT*>(&wq[i]);
#pragma unroll
            for (int k = 0; k < VW; ++k) acc[i] = fmaf(uv[k], to_f<IT>(e[k]), acc[i]);
          }
        }
      }
      for (int c = (vec_ok ? nvec * VW : 0) + lane; c < len; c += 32) {
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i] = fmaf(u_s[c], to_f<IT>(wr[i][c]), acc[i]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float t = mix_warp_sum(acc[i]);
        if (lane == 0 && j0 + i < J) part[j0 + i] = t;
      }
    }
  }
  cluster.sync();  // every CTA's partials are written
  for (int j = tid; j < J; j += kMixThreads) {
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < CL; ++r) s += cluster.map_shared_rank(part, r)[j];
    dbl[j] = to_f<IT>(from_f<IT>(s));
  }
  cluster.sync();  // the remote reads are done (CTAs may exit after this) and dbl is visible

  // 3. SSM step of this CTA's channels: TPC lanes per channel, R chunks of 4 states per lane
  const int DR = a.dt_rank;
  const float* Bv = dbl + DR;
  const float* Cv = dbl + DR + N;
  const int q = tid % TPC;
  for (int base = c_begin; base < c_end; base += kMixThreads / TPC) {
    const int c = base + tid / TPC;
    const bool ok = c < c_end;
    const int cc = ok ? c : c_begin;
    // the state and A loads do not depend on dt: issue them first
    float* st = a.ssm_state + ((int64_t)b * d + cc) * N;
    const bool vec = P.vec_a != 0;
    float s[R][kSPW], av[R][kSPW];
#pragma unroll
    for (int rr = 0; rr < R; ++rr) {
      const int nb = 4 * (q + TPC * rr);
      if (vec && nb < N) {
        const float4 v = *reinterpret_cast<const float4*>(st + nb);
        const float4 w = *reinterpret_cast<const float4*>(a.A + (int64_t)cc * N + nb);
        s[rr][0] = v.x; s[rr][1] = v.y; s[rr][2] = v.z; s[rr][3] = v.w;
        av[rr][0] = w.x; av[rr][1] = w.y; av[rr][2] = w.z; av[rr][3] = w.w;
      } else {
#pragma unroll
        for (int j = 0; j < kSPW; ++j) {
          s[rr][j] = (nb + j < N) ? st[nb + j] : 0.f;
          av[rr][j] = (nb + j < N) ? a.A[(int64_t)cc * N + nb + j] : 0.f;
        }
      }
    }
    // delta projection: the channel's TPC lanes split the dt_rank-long dot product
    const IT* wrow = (const IT*)a.dt_proj + (int64_t)cc * DR;
    float dv = 0.f, d1 = 0.f;
    int r = q;
#pragma unroll 4
    for (; r + TPC < DR; r += 2 * TPC) {
      dv = fmaf(dbl[r], to_f<IT>(wrow[r]), dv);
      d1 = fmaf(dbl[r + TPC], to_f<IT>(wrow[r + TPC]), d1);
    }
    if (r < DR) dv = fmaf(dbl[r], to_f<IT>(wrow[r]), dv);
    dv += d1;
#pragma unroll
    for (int o = 1; o < TPC; o <<= 1) dv += __shfl_xor_sync(0xffffffffu, dv, o);
    if (a.dt_bias != nullptr) dv += a.dt_bias[cc];
    const float dt = a.dt_softplus ? softplus_thr(dv) : dv;
    const float uv = u_s[cc - c_begin];
    float y = 0.f;
    if (ok) {
#pragma unroll
      for (int rr = 0; rr < R; ++rr) {
        const int nb = 4 * (q + TPC * rr);
#pragma unroll
        for (int j = 0; j < kSPW; ++j) {
          const int n = nb + j;
          if (n < N) {
            s[rr][j] = fmaf(exp_fast(dt * av[rr][j]), s[rr][j], dt * uv * Bv[n]);
            y = fmaf(Cv[n], s[rr][j], y);
          }
        }
        if (vec && nb < N) {
          *reinterpret_cast<float4*>(st + nb) = make_float4(s[rr][0], s[rr][1], s[rr][2], s[rr][3]);
        } else {
#pragma unroll
          for (int j = 0; j < kSPW; ++j)
            if (nb + j < N) st[nb + j] = s[rr][j];
        }
      }
    }
#pragma unroll
    for (int o = 1; o < TPC; o <<= 1) y += __shfl_xor_sync(0xffffffffu, y, o);
    if (ok && q == 0) {
      if (a.D != nullptr) y = fmaf(a.D[c], uv, y);
      const float zv = to_f<IT>(xb[d + c]);
      y *= zv * sigmoid_fast(zv);
      ((IT*)a.y)[(int64_t)b * a.y_batch_stride + c] = from_f<IT>(y);
    }
  }
}

}  // namespace ssb
