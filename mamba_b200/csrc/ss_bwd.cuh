// Backward selective scan for sm_100a.
//
// Gradients (reference backward_kernel.cu:320-585, same symbols as the forward):
//   dy_t        = dout_t [* silu(z_t)]                         (gate of mamba_simple.py:143-146)
//   dh_t[n]     = C_t[n] dy_t + exp(delta'_{t+1} A[n]) dh_{t+1}[n]       (reverse recurrence)
//   g_t[n]      = dh_t[n] * exp(delta'_t A[n]) * h_{t-1}[n]
//   du_t        = D dy_t + delta'_t * sum_n B_t[n] dh_t[n]
//   ddelta'_t   = sum_n A[n] g_t[n] + u_t * sum_n B_t[n] dh_t[n]
//   ddelta_t    = ddelta'_t * sigmoid(delta_t + bias)  where delta_t + bias <= 20 (softplus)
//   dA[n]      += delta'_t g_t[n];  dD += dy_t u_t;  dbias += ddelta_t
//   dB_t[n]    += dh_t[n] delta'_t u_t     (summed over the channels of the group)
//   dC_t[n]    += dy_t h_t[n]              (summed over the channels of the group)
//   dz_t        = dout_t * y_t * silu'(z_t)
//
// Same CTA shape as the forward (lane = channel, warp = 4 states).  Tiles of 16 steps are
// visited last to first.  For each tile a lane
//   * restarts its 4 states from the forward's checkpoint of the previous tile boundary,
//   * runs the 16 forward steps keeping exp(delta'A) and h_{t-1} in registers (128 values),
//   * runs the 16 reverse steps, carrying dh across tiles in registers,
//   * reduces its dB / dC contributions over the warp's 32 channels with a butterfly
//     transpose (each lane ends with 4 consecutive steps of one (B|C, n) row) and adds them
//     to global memory with one 16-byte vector reduction per lane — instead of the
//     reference's two fp32 atomics per element and state (backward_kernel.cu:466-478);
//   * leaves the per-step sums over its states (for du, ddelta, dz) in shared memory, where
//     the element phase combines the warps.
// Inputs (u, delta, dout, z, the B / C tiles and the checkpointed states) stream through a
// TMA ring of kStages tiles, as in the forward; kTMA = false loads each tile synchronously.
#pragma once
#include "ss_common.cuh"

namespace ssb {

template <typename IT, int kNW, bool kVarB, bool kVarC, bool kHasZ>
struct BwdSmem {
  static constexpr int NS = kSPW * kNW;
  alignas(128) IT u[kStages][kCh][kTile];
  alignas(128) IT d[kStages][kCh][kTile];
  alignas(128) IT g[kStages][kCh][kTile];
  alignas(128) IT z[kHasZ ? kStages : 1][kCh][kTile];
  alignas(128) float Braw[kVarB ? kStages : 1][NS * kTile];
  alignas(128) float Craw[kVarC ? kStages : 1][NS * kTile];
  alignas(128) float hck[kStages][NS][kCh];   // states at the tile start, [n][channel]
  alignas(16) float4 dt_s[kCh][4];
  alignas(16) float4 dtu_s[kCh][4];
  alignas(16) float4 dy_s[kCh][4];
  alignas(16) float4 sig_s[kCh][4];
  alignas(16) float4 gz_s[kHasZ ? kCh : 1][4];
  alignas(16) float B_s[kVarB ? kTile : 1][NS];
  alignas(16) float C_s[kVarC ? kTile : 1][NS];
  float s1_s[kNW][kTile][kPad];
  float s2_s[kNW][kTile][kPad];
  float y_s[kHasZ ? kNW : 1][kTile][kPad];
  alignas(8) uint64_t full[kStages];
};

template <typename IT, int kNW, bool kVarB, bool kVarC, bool kHasZ, bool kTMA>
__global__ void __launch_bounds__(32 * kNW, 2) ss_bwd_kernel(const __grid_constant__ BwdK P) {
  constexpr int NT = 32 * kNW;
  constexpr int NS = kSPW * kNW;
  constexpr int S = kTile / kNW;
  constexpr int KV = (kVarB ? 64 : 0) + (kVarC ? 64 : 0);   // butterfly values per lane
  using Sm = BwdSmem<IT, kNW, kVarB, kVarC, kHasZ>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Sm& sm = *reinterpret_cast<Sm*>(smem_raw);
  const ss_bwd_args& a = P.a;
  const ss_fwd_args& f = a.f;

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int grp = blockIdx.x / P.tpg;
  const int cl0 = (blockIdx.x % P.tpg) * kCh;
  const int c0 = grp * P.dpg + cl0;
  const int nvalid = min(kCh, P.dpg - cl0);
  const int b = blockIdx.y;
  const int N = f.dstate, L = f.seqlen;
  const bool bc_f32 = f.bc_dtype == SS_F32;

  // ---- scan role
  const bool lane_ok = lane < nvalid;
  const int c = c0 + lane;
  float A2[kSPW], Ad[kSPW], Bc[kSPW], Cc[kSPW];
  float dAacc[kSPW], e[kSPW], dBc[kSPW], dCc[kSPW];
#pragma unroll
  for (int j = 0; j < kSPW; ++j) {
    const int n = kSPW * w + j;
    const bool ok = lane_ok && n < N;
    const int64_t ia = (int64_t)c * N + n;
    Ad[j] = ok ? f.A[ia] : 0.f;
    A2[j] = Ad[j] * kLog2e;
    Bc[j] = 0.f;
    Cc[j] = 0.f;
    if (!kVarB && ok) Bc[j] = bc_f32 ? ((const float*)f.B)[ia] : to_f<IT>(((const IT*)f.B)[ia]);
    if (!kVarC && ok) Cc[j] = bc_f32 ? ((const float*)f.C)[ia] : to_f<IT>(((const IT*)f.C)[ia]);
    dAacc[j] = 0.f;
    e[j] = 0.f;
    dBc[j] = 0.f;
    dCc[j] = 0.f;
  }

  // ---- element role
  const int pc = tid / kNW, pq = tid % kNW;
  const bool pc_ok = pc < nvalid;
  const float Dv = (f.D != nullptr && pc_ok) ? f.D[c0 + pc] : 0.f;
  const float bias = (f.delta_bias != nullptr && pc_ok) ? f.delta_bias[c0 + pc] : 0.f;
  float dD_acc = 0.f, db_acc = 0.f;

  const IT* ub = (const IT*)f.u + (int64_t)b * f.u_batch_stride + (int64_t)c0 * f.u_dim_stride;
  const IT* db = (const IT*)f.delta + (int64_t)b * f.delta_batch_stride + (int64_t)c0 * f.delta_dim_stride;
  const IT* gb = (const IT*)a.dout + (int64_t)b * a.dout_batch_stride + (int64_t)c0 * a.dout_dim_stride;
  const IT* zb = kHasZ ? (const IT*)f.z + (int64_t)b * f.z_batch_stride + (int64_t)c0 * f.z_dim_stride : nullptr;
  IT* du_row = (IT*)a.du + (int64_t)b * a.du_batch_stride + (int64_t)(c0 + pc) * a.du_dim_stride;
  IT* dd_row = (IT*)a.ddelta + (int64_t)b * a.ddelta_batch_stride + (int64_t)(c0 + pc) * a.ddelta_dim_stride;
  IT* dz_row = kHasZ ? (IT*)a.dz + (int64_t)b * a.dz_batch_stride + (int64_t)(c0 + pc) * a.dz_dim_stride : nullptr;
  const int64_t bc_off = ((int64_t)b * f.ngroups + grp) * N * (int64_t)L;

  const int ntiles = P.ntiles;
  const uint32_t io_bytes = kCh * kTile * (uint32_t)sizeof(IT);
  const uint32_t bc_bytes = NS * kTile * (bc_f32 ? 4u : (uint32_t)sizeof(IT));
  const uint32_t h_bytes = NS * kCh * 4u;
  // iteration i handles tile ntiles-1-i
  auto issue = [&](int i, int s) {
    const int k = ntiles - 1 - i;
    uint64_t* bar = &sm.full[s];
    const uint32_t bytes = (3 + (kHasZ ? 1 : 0)) * io_bytes + ((kVarB ? 1 : 0) + (kVarC ? 1 : 0)) * bc_bytes +
                           (k > 0 ? h_bytes : 0u);
    mbar_expect_tx(bar, bytes);
    const int t0 = k * kTile;
    tma_load_3d(&sm.u[s][0][0], &P.tm_u, t0, c0, b, bar);
    tma_load_3d(&sm.d[s][0][0], &P.tm_d, t0, c0, b, bar);
    tma_load_3d(&sm.g[s][0][0], &P.tm_g, t0, c0, b, bar);
    if constexpr (kHasZ) tma_load_3d(&sm.z[s][0][0], &P.tm_z, t0, c0, b, bar);
    if constexpr (kVarB) tma_load_3d(&sm.Braw[s][0], &P.tm_B, t0, 0, b * f.ngroups + grp, bar);
    if constexpr (kVarC) tma_load_3d(&sm.Craw[s][0], &P.tm_C, t0, 0, b * f.ngroups + grp, bar);
    if (k > 0) tma_load_3d(&sm.hck[s][0][0], &P.tm_h, c0, 0, b * ntiles + (k - 1), bar);
  };
  if constexpr (kTMA) {
    if (tid == 0) {
      for (int s = 0; s < kStages; ++s) mbar_init(&sm.full[s], 1);
      mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0)
      for (int s = 0; s < kStages && s < ntiles; ++s) issue(s, s);
  }

  for (int it = 0; it < ntiles; ++it) {
    const int k = ntiles - 1 - it;
    const int t0 = k * kTile;
    const int tlen = min(kTile, L - t0);
    const int stg = kTMA ? it % kStages : 0;
    bool failed = false;
    float hp[kTile + 1][kSPW];
    if constexpr (kTMA) {
      failed = !mbar_wait_bounded(&sm.full[stg], (it / kStages) & 1);
      if constexpr (kVarB) widen_bc<IT, NT, NS>(sm.B_s, sm.Braw[stg], bc_f32);
      if constexpr (kVarC) widen_bc<IT, NT, NS>(sm.C_s, sm.Craw[stg], bc_f32);
#pragma unroll
      for (int j = 0; j < kSPW; ++j) hp[0][j] = (k > 0) ? sm.hck[stg][kSPW * w + j][lane] : 0.f;
    } else {
      load_tile<IT, NT>(sm.u[0], ub + t0, f.u_dim_stride, nvalid, tlen, P.vec_u);
      load_tile<IT, NT>(sm.d[0], db + t0, f.delta_dim_stride, nvalid, tlen, P.vec_d);
      load_tile<IT, NT>(sm.g[0], gb + t0, a.dout_dim_stride, nvalid, tlen, P.vec_dout);
      if constexpr (kHasZ) load_tile<IT, NT>(sm.z[0], zb + t0, f.z_dim_stride, nvalid, tlen, P.vec_z);
      if constexpr (kVarB) {
        if (bc_f32) load_bc_tile<float, NT, NS>(sm.B_s, (const float*)f.B + bc_off + t0, L, N, tlen);
        else load_bc_tile<IT, NT, NS>(sm.B_s, (const IT*)f.B + bc_off + t0, L, N, tlen);
      }
      if constexpr (kVarC) {
        if (bc_f32) load_bc_tile<float, NT, NS>(sm.C_s, (const float*)f.C + bc_off + t0, L, N, tlen);
        else load_bc_tile<IT, NT, NS>(sm.C_s, (const IT*)f.C + bc_off + t0, L, N, tlen);
      }
      // states at the tile start (end of the previous tile), from the forward's checkpoints
#pragma unroll
      for (int j = 0; j < kSPW; ++j) {
        const int n = kSPW * w + j;
        hp[0][j] = (k > 0 && lane_ok && n < N)
                       ? f.ckpt[(((int64_t)b * ntiles + (k - 1)) * N + n) * f.dim + c]
                       : 0.f;
      }
      __syncthreads();
    }

    // ---- element phase 1: delta', delta'u, dy, softplus slope, gate slope
    {
      float dtv[S], dtuv[S], dyv[S], sgv[S], gzv[S];
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const int t = pq * S + i;
        const bool ok = pc_ok && t < tlen;
        const float uv = to_f<IT>(sm.u[stg][pc][t]);
        const float v = to_f<IT>(sm.d[stg][pc][t]) + bias;
        float dt = v, sg = 1.f;
        if (f.delta_softplus && v <= 20.f) {
          dt = log1pf(exp_fast(v));
          sg = sigmoid_fast(v);
        }
        const float go = to_f<IT>(sm.g[stg][pc][t]);
        float dy = go, gz = 0.f;
        if constexpr (kHasZ) {
          const float zv = to_f<IT>(sm.z[stg][pc][t]);
          const float sz = sigmoid_fast(zv);
          dy = go * zv * sz;
          gz = go * sz * (1.f + zv * (1.f - sz));
        }
        if (!ok) {
          dt = 0.f;
          dy = 0.f;
        }
        dD_acc = fmaf(dy, uv, dD_acc);
        dtv[i] = dt;
        dtuv[i] = dt * uv;
        dyv[i] = dy;
        sgv[i] = sg;
        gzv[i] = gz;
      }
#pragma unroll
      for (int q = 0; q < S / 4; ++q) {
        const int ch = swz(pc, pq * (S / 4) + q);
        sm.dt_s[pc][ch] = make_float4(dtv[4 * q], dtv[4 * q + 1], dtv[4 * q + 2], dtv[4 * q + 3]);
        sm.dtu_s[pc][ch] = make_float4(dtuv[4 * q], dtuv[4 * q + 1], dtuv[4 * q + 2], dtuv[4 * q + 3]);
        sm.dy_s[pc][ch] = make_float4(dyv[4 * q], dyv[4 * q + 1], dyv[4 * q + 2], dyv[4 * q + 3]);
        sm.sig_s[pc][ch] = make_float4(sgv[4 * q], sgv[4 * q + 1], sgv[4 * q + 2], sgv[4 * q + 3]);
        if constexpr (kHasZ)
          sm.gz_s[pc][ch] = make_float4(gzv[4 * q], gzv[4 * q + 1], gzv[4 * q + 2], gzv[4 * q + 3]);
      }
    }
    if (__syncthreads_or(failed)) {
      if (tid == 0) {
        if (P.status != nullptr) atomicOr(P.status, kStatusTimeout);
        for (int j = it + 1; j < ntiles && j < it + kStages; ++j)
          mbar_wait_bounded(&sm.full[j % kStages], (j / kStages) & 1);
      }
      __syncthreads();
      return;
    }

    // ---- scan phase, forward: decays and states of the tile in registers
    float da[kTile][kSPW];
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
      const float4 dt4 = sm.dt_s[lane][swz(lane, i4)];
      const float4 du4 = sm.dtu_s[lane][swz(lane, i4)];
      const float dts[4] = {dt4.x, dt4.y, dt4.z, dt4.w};
      const float dus[4] = {du4.x, du4.y, du4.z, du4.w};
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const int t = 4 * i4 + s;
        float Bv[kSPW];
        if constexpr (kVarB) {
          const float4 q = *reinterpret_cast<const float4*>(&sm.B_s[t][kSPW * w]);
          Bv[0] = q.x; Bv[1] = q.y; Bv[2] = q.z; Bv[3] = q.w;
        } else {
#pragma unroll
          for (int j = 0; j < kSPW; ++j) Bv[j] = Bc[j];
        }
#pragma unroll
        for (int j = 0; j < kSPW; ++j) {
          da[t][j] = ex2(dts[s] * A2[j]);
          hp[t + 1][j] = fmaf(da[t][j], hp[t][j], dus[s] * Bv[j]);
        }
        if constexpr (kHasZ) {
          float Cv[kSPW];
          if constexpr (kVarC) {
            const float4 q = *reinterpret_cast<const float4*>(&sm.C_s[t][kSPW * w]);
            Cv[0] = q.x; Cv[1] = q.y; Cv[2] = q.z; Cv[3] = q.w;
          } else {
#pragma unroll
            for (int j = 0; j < kSPW; ++j) Cv[j] = Cc[j];
          }
          float yp = 0.f;
#pragma unroll
          for (int j = 0; j < kSPW; ++j) yp = fmaf(Cv[j], hp[t + 1][j], yp);
          sm.y_s[w][t][lane] = yp;
        }
      }
    }

    // ---- scan phase, reverse.  The dB / dC contributions of each step are folded across
    //      the warp's lanes right away (the first three butterfly stages pair values of the
    //      same step), leaving one partial per lane and step in W[t].
    float W[kTile];
#pragma unroll
    for (int i4 = 3; i4 >= 0; --i4) {
      const float4 dt4 = sm.dt_s[lane][swz(lane, i4)];
      const float4 du4 = sm.dtu_s[lane][swz(lane, i4)];
      const float4 dy4 = sm.dy_s[lane][swz(lane, i4)];
      const float dts[4] = {dt4.x, dt4.y, dt4.z, dt4.w};
      const float dus[4] = {du4.x, du4.y, du4.z, du4.w};
      const float dys[4] = {dy4.x, dy4.y, dy4.z, dy4.w};
#pragma unroll
      for (int s = 3; s >= 0; --s) {
        const int t = 4 * i4 + s;
        float Bv[kSPW], Cv[kSPW];
        if constexpr (kVarB) {
          const float4 q = *reinterpret_cast<const float4*>(&sm.B_s[t][kSPW * w]);
          Bv[0] = q.x; Bv[1] = q.y; Bv[2] = q.z; Bv[3] = q.w;
        } else {
#pragma unroll
          for (int j = 0; j < kSPW; ++j) Bv[j] = Bc[j];
        }
        if constexpr (kVarC) {
          const float4 q = *reinterpret_cast<const float4*>(&sm.C_s[t][kSPW * w]);
          Cv[0] = q.x; Cv[1] = q.y; Cv[2] = q.z; Cv[3] = q.w;
        } else {
#pragma unroll
          for (int j = 0; j < kSPW; ++j) Cv[j] = Cc[j];
        }
        float s1 = 0.f, s2 = 0.f, vB[kSPW], vC[kSPW];
#pragma unroll
        for (int j = 0; j < kSPW; ++j) {
          const float dh = fmaf(Cv[j], dys[s], e[j]);
          const float ee = da[t][j] * dh;
          const float g = ee * hp[t][j];
          dAacc[j] = fmaf(dts[s], g, dAacc[j]);
          s1 = fmaf(Ad[j], g, s1);
          s2 = fmaf(Bv[j], dh, s2);
          vB[j] = dh * dus[s];
          vC[j] = dys[s] * hp[t + 1][j];
          if constexpr (!kVarB) dBc[j] = fmaf(dh, dus[s], dBc[j]);
          if constexpr (!kVarC) dCc[j] = fmaf(dys[s], hp[t + 1][j], dCc[j]);
          e[j] = ee;
        }
        sm.s1_s[w][t][lane] = s1;
        sm.s2_s[w][t][lane] = s2;
        if constexpr (KV == 128) W[t] = fold_step_bc(vB, vC, lane);
        else if constexpr (kVarB) W[t] = fold_step_one(vB, lane);
        else if constexpr (kVarC) W[t] = fold_step_one(vC, lane);
      }
    }

    // ---- dB / dC of this tile: reduce over the warp's channels, one vector add per lane
    if constexpr (KV > 0) {
      float V[KV / 32];
      fold_tile<KV / 32>(W, V, lane);
      constexpr int PER = KV / 32;                 // 4 (both variable) or 2
      const int type = (KV == 128) ? (lane >> 4) : (kVarB ? 0 : 1);
      const int j = (KV == 128) ? ((lane >> 2) & 3) : (lane >> 3);
      const int tt = (KV == 128) ? 4 * (lane & 3) : 2 * (lane & 7);
      const int n = kSPW * w + j;
      if (n < N) {
        float* dst = (type == 0 ? a.dB : a.dC) + bc_off + (int64_t)n * L + t0 + tt;
        if (P.vec_dbc && tt + PER <= tlen) {
          if constexpr (PER == 4) red_add_v4(dst, V[0], V[1], V[2], V[3]);
          else red_add_v2(dst, V[0], V[1]);
        } else {
#pragma unroll
          for (int i = 0; i < PER; ++i)
            if (tt + i < tlen) red_add(dst + i, V[i]);
        }
      }
    }
    // carry for the next (earlier) tile: e = exp(delta'_{t0} A) dh_{t0} is already in e[]
    __syncthreads();

    // ---- element phase 2: du, ddelta, dz
    {
      float duv[S], ddv[S], dzv[S];
#pragma unroll
      for (int q = 0; q < S / 4; ++q) {
        const int ch = swz(pc, pq * (S / 4) + q);
        const float4 dt4 = sm.dt_s[pc][ch], dy4 = sm.dy_s[pc][ch], sg4 = sm.sig_s[pc][ch];
        float4 gz4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if constexpr (kHasZ) gz4 = sm.gz_s[pc][ch];
        const float dts[4] = {dt4.x, dt4.y, dt4.z, dt4.w};
        const float dys[4] = {dy4.x, dy4.y, dy4.z, dy4.w};
        const float sgs[4] = {sg4.x, sg4.y, sg4.z, sg4.w};
        const float gzs[4] = {gz4.x, gz4.y, gz4.z, gz4.w};
#pragma unroll
        for (int r = 0; r < 4; ++r) {
          const int i = 4 * q + r;
          const int t = pq * S + i;
          float S1 = 0.f, S2 = 0.f, yv = 0.f;
#pragma unroll
          for (int g = 0; g < kNW; ++g) {
            S1 += sm.s1_s[g][t][pc];
            S2 += sm.s2_s[g][t][pc];
            if constexpr (kHasZ) yv += sm.y_s[g][t][pc];
          }
          const float uv = to_f<IT>(sm.u[stg][pc][t]);
          duv[i] = fmaf(Dv, dys[r], dts[r] * S2);
          const float dd = fmaf(uv, S2, S1) * sgs[r];
          ddv[i] = dd;
          if (pc_ok && t < tlen) db_acc += dd;
          if constexpr (kHasZ) dzv[i] = gzs[r] * fmaf(Dv, uv, yv);
        }
      }
      const int nv = pc_ok ? max(0, min(S, tlen - pq * S)) : 0;
      store_run<IT, S>(du_row + t0 + pq * S, duv, nv, P.vec_du);
      store_run<IT, S>(dd_row + t0 + pq * S, ddv, nv, P.vec_dd);
      if constexpr (kHasZ) store_run<IT, S>(dz_row + t0 + pq * S, dzv, nv, P.vec_dz);
    }
    __syncthreads();
    if constexpr (kTMA) {
      if (tid == 0 && it + kStages < ntiles) issue(it + kStages, stg);
    }
  }

  // ---- per-channel parameter gradients (summed over batch rows by the atomics)
#pragma unroll
  for (int j = 0; j < kSPW; ++j) {
    const int n = kSPW * w + j;
    if (lane_ok && n < N) {
      const int64_t ia = (int64_t)c * N + n;
      red_add(a.dA + ia, dAacc[j]);
      if constexpr (!kVarB) red_add(a.dB + ia, dBc[j]);
      if constexpr (!kVarC) red_add(a.dC + ia, dCc[j]);
    }
  }
  // the kNW element-role threads of a channel are adjacent lanes
#pragma unroll
  for (int o = 1; o < kNW; o <<= 1) {
    dD_acc += __shfl_xor_sync(0xffffffffu, dD_acc, o);
    db_acc += __shfl_xor_sync(0xffffffffu, db_acc, o);
  }
  if (pq == 0 && pc_ok) {
    if (a.dD != nullptr) red_add(a.dD + c0 + pc, dD_acc);
    if (a.ddelta_bias != nullptr) red_add(a.ddelta_bias + c0 + pc, db_acc);
  }
}

}  // namespace ssb
