// Forward selective scan for sm_100a.
//
// Computes, per (batch b, channel c) row and state n (reference forward_kernel.cu:213-293):
//   delta'_t = softplus(delta_t + bias_c)  (threshold 20)        [or delta_t + bias_c]
//   h_t[n]   = exp(delta'_t * A[c,n]) * h_{t-1}[n] + delta'_t * u_t * B_t[n]
//   y_t      = D_c * u_t + sum_n C_t[n] * h_t[n]
//   out_t    = y_t * silu(z_t)   when z is given (modules/mamba_simple.py:143-146)
//
// CTA = (32 channels of one group, one batch row); lane = channel, warp w = states 4w..4w+3.
// Per 16-step tile:
//   1. u, delta, z tiles (32 x 16) and the variable B / C tiles (16 x dstate) are staged in
//      shared memory with 16-byte vector loads (B and C once per CTA for all 32 channels);
//   2. each element's delta' and delta'*u is computed once (one thread per element run)
//      and stored as fp32;
//   3. every lane advances its 4 states through the 16 steps in registers — one ex2, one
//      FMUL, two FFMA per (element, state); the partial sum over its 4 states of C*h goes
//      to shared memory;
//   4. the warps' partial sums are added, D*u and the gate applied, and the tile stored.
// At each tile end the 4 states of every lane go to the checkpoint buffer
// ckpt[b][tile][n][c] (coalesced over channels); the last tile's entry is the final state.
#pragma once
#include "ss_common.cuh"

namespace ssb {

template <typename IT, int kNW, bool kVarB, bool kVarC, bool kHasZ>
__global__ void __launch_bounds__(32 * kNW, 4) ss_fwd_kernel(const __grid_constant__ FwdK P) {
  constexpr int NT = 32 * kNW;
  constexpr int NS = kSPW * kNW;   // states covered by the CTA (dstate padded up)
  constexpr int S = kTile / kNW;   // steps per thread in the element-wise phases
  const ss_fwd_args& a = P.a;

  __shared__ __align__(16) IT u_raw[kCh][kTile];
  __shared__ __align__(16) IT d_raw[kCh][kTile];
  __shared__ __align__(16) IT z_raw[kHasZ ? kCh : 1][kTile];
  __shared__ float4 dt_s[kCh][4];
  __shared__ float4 dtu_s[kCh][4];
  __shared__ __align__(16) float B_s[kVarB ? kTile : 1][NS];
  __shared__ __align__(16) float C_s[kVarC ? kTile : 1][NS];
  __shared__ float y_s[kNW][kTile][kPad];

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int grp = blockIdx.x / P.tpg;
  const int cl0 = (blockIdx.x % P.tpg) * kCh;
  const int c0 = grp * P.dpg + cl0;
  const int nvalid = min(kCh, P.dpg - cl0);
  const int b = blockIdx.y;
  const int N = a.dstate, L = a.seqlen;
  const bool bc_f32 = a.bc_dtype == SS_F32;

  // ---- scan role: channel c0 + lane, states kSPW*w + j
  const bool lane_ok = lane < nvalid;
  const int c = c0 + lane;
  float A2[kSPW], Bc[kSPW], Cc[kSPW], h[kSPW];
#pragma unroll
  for (int j = 0; j < kSPW; ++j) {
    const int n = kSPW * w + j;
    const bool ok = lane_ok && n < N;
    const int64_t ia = (int64_t)c * N + n;
    A2[j] = ok ? a.A[ia] * kLog2e : 0.f;
    Bc[j] = 0.f;
    Cc[j] = 0.f;
    if (!kVarB && ok) Bc[j] = bc_f32 ? ((const float*)a.B)[ia] : to_f<IT>(((const IT*)a.B)[ia]);
    if (!kVarC && ok) Cc[j] = bc_f32 ? ((const float*)a.C)[ia] : to_f<IT>(((const IT*)a.C)[ia]);
    h[j] = 0.f;
  }

  // ---- element role: channel c0 + pc, steps pq*S .. pq*S + S - 1 of each tile
  const int pc = tid / kNW, pq = tid % kNW;
  const bool pc_ok = pc < nvalid;
  const float Dv = (a.D != nullptr && pc_ok) ? a.D[c0 + pc] : 0.f;
  const float bias = (a.delta_bias != nullptr && pc_ok) ? a.delta_bias[c0 + pc] : 0.f;

  const IT* ub = (const IT*)a.u + (int64_t)b * a.u_batch_stride + (int64_t)c0 * a.u_dim_stride;
  const IT* db = (const IT*)a.delta + (int64_t)b * a.delta_batch_stride + (int64_t)c0 * a.delta_dim_stride;
  const IT* zb = kHasZ ? (const IT*)a.z + (int64_t)b * a.z_batch_stride + (int64_t)c0 * a.z_dim_stride : nullptr;
  IT* orow = (IT*)a.out + (int64_t)b * a.out_batch_stride + (int64_t)(c0 + pc) * a.out_dim_stride;
  const int64_t bc_off = ((int64_t)b * a.ngroups + grp) * N * (int64_t)L;

  for (int k = 0; k < P.ntiles; ++k) {
    const int t0 = k * kTile;
    const int tlen = min(kTile, L - t0);
    load_tile<IT, NT>(u_raw, ub + t0, a.u_dim_stride, nvalid, tlen, P.vec_u);
    load_tile<IT, NT>(d_raw, db + t0, a.delta_dim_stride, nvalid, tlen, P.vec_d);
    if constexpr (kHasZ) load_tile<IT, NT>(z_raw, zb + t0, a.z_dim_stride, nvalid, tlen, P.vec_z);
    if constexpr (kVarB) {
      if (bc_f32) load_bc_tile<float, NT, NS>(B_s, (const float*)a.B + bc_off + t0, L, N, tlen);
      else load_bc_tile<IT, NT, NS>(B_s, (const IT*)a.B + bc_off + t0, L, N, tlen);
    }
    if constexpr (kVarC) {
      if (bc_f32) load_bc_tile<float, NT, NS>(C_s, (const float*)a.C + bc_off + t0, L, N, tlen);
      else load_bc_tile<IT, NT, NS>(C_s, (const IT*)a.C + bc_off + t0, L, N, tlen);
    }
    __syncthreads();

    // ---- 2. delta' and delta'*u, once per element (steps past seqlen get delta' = 0,
    //         so the states pass through them unchanged)
    {
      float dtv[S], dtuv[S];
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const int t = pq * S + i;
        const bool ok = pc_ok && t < tlen;
        const float uv = to_f<IT>(u_raw[pc][t]);
        const float v = to_f<IT>(d_raw[pc][t]) + bias;
        float dt = a.delta_softplus ? softplus_thr(v) : v;
        dt = ok ? dt : 0.f;
        dtv[i] = dt;
        dtuv[i] = dt * uv;
      }
#pragma unroll
      for (int q = 0; q < S / 4; ++q) {
        const int ch = swz(pc, pq * (S / 4) + q);
        dt_s[pc][ch] = make_float4(dtv[4 * q], dtv[4 * q + 1], dtv[4 * q + 2], dtv[4 * q + 3]);
        dtu_s[pc][ch] = make_float4(dtuv[4 * q], dtuv[4 * q + 1], dtuv[4 * q + 2], dtuv[4 * q + 3]);
      }
    }
    __syncthreads();

    // ---- 3. the recurrence, 4 states per lane, 16 steps
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
      const float4 dt4 = dt_s[lane][swz(lane, i4)];
      const float4 du4 = dtu_s[lane][swz(lane, i4)];
      const float dts[4] = {dt4.x, dt4.y, dt4.z, dt4.w};
      const float dus[4] = {du4.x, du4.y, du4.z, du4.w};
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int t = 4 * i4 + s;
        float Bv[kSPW], Cv[kSPW];
        if constexpr (kVarB) {
          const float4 q = *reinterpret_cast<const float4*>(&B_s[t][kSPW * w]);
          Bv[0] = q.x; Bv[1] = q.y; Bv[2] = q.z; Bv[3] = q.w;
        } else {
#pragma unroll
          for (int j = 0; j < kSPW; ++j) Bv[j] = Bc[j];
        }
        if constexpr (kVarC) {
          const float4 q = *reinterpret_cast<const float4*>(&C_s[t][kSPW * w]);
          Cv[0] = q.x; Cv[1] = q.y; Cv[2] = q.z; Cv[3] = q.w;
        } else {
#pragma unroll
          for (int j = 0; j < kSPW; ++j) Cv[j] = Cc[j];
        }
        float yp = 0.f;
#pragma unroll
        for (int j = 0; j < kSPW; ++j) {
          const float da = ex2(dts[s] * A2[j]);
          h[j] = fmaf(da, h[j], dus[s] * Bv[j]);
          yp = fmaf(Cv[j], h[j], yp);
        }
        y_s[w][t][lane] = yp;
      }
    }
    if (a.ckpt != nullptr && lane_ok) {
      float* ck = a.ckpt + ((int64_t)b * P.ntiles + k) * N * (int64_t)a.dim + c;
#pragma unroll
      for (int j = 0; j < kSPW; ++j) {
        const int n = kSPW * w + j;
        if (n < N) ck[(int64_t)n * a.dim] = h[j];
      }
    }
    __syncthreads();

    // ---- 4. combine the warps' partial sums, add D*u, gate, store
    {
      float yv[S];
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const int t = pq * S + i;
        float y = Dv * to_f<IT>(u_raw[pc][t]);
#pragma unroll
        for (int g = 0; g < kNW; ++g) y += y_s[g][t][pc];
        if constexpr (kHasZ) {
          const float zv = to_f<IT>(z_raw[pc][t]);
          y *= zv * sigmoid_fast(zv);
        }
        yv[i] = y;
      }
      const int nv = pc_ok ? max(0, min(S, tlen - pq * S)) : 0;
      store_run<IT, S>(orow + t0 + pq * S, yv, nv, P.vec_out);
    }
    __syncthreads();
  }

  if (a.last_state != nullptr && lane_ok) {
    float* ls = a.last_state + ((int64_t)b * a.dim + c) * N;
#pragma unroll
    for (int j = 0; j < kSPW; ++j) {
      const int n = kSPW * w + j;
      if (n < N) ls[n] = h[j];
    }
  }
}

}  // namespace ssb
