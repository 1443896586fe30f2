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
// Same CTA shape as the forward (lane = channel, warp = 4 states, handled as two pairs
// with packed fp32x2 arithmetic).  Tiles of 16 steps are visited last to first.  Per tile a
// lane
//   * restarts its 4 states from the forward's checkpoint of the previous tile boundary,
//   * runs the 16 forward steps keeping h_{t-1} in registers (exp(delta'A) is recomputed
//     in the reverse steps rather than kept: registers, not MUFU, are the scarce resource),
//   * runs the 16 reverse steps, carrying dh across tiles in registers,
//   * hands its dB / dC contributions to a per-warp shared-memory block every 4 steps; the
//     warp then sums them over its 32 channels (each lane one (step, B|C, state-pair) row,
//     16-byte reads) and, once per tile, adds 4 consecutive steps of one (B|C, n) row to
//     global memory with a 16-byte vector reduction — instead of the reference's two fp32
//     atomics per element and state (backward_kernel.cu:466-478);
//   * leaves the per-step sums over its states (for du, ddelta) in shared memory, where the
//     element phase combines the warps (dz uses the ungated y the forward saved).
// Inputs (u, delta, dout, z, y, the B / C tiles and the checkpointed states) stream through
// a TMA ring of kStagesBwd tiles; kTMA = false loads each tile synchronously.  Shared memory
// is kept under ~72 KB (bf16) so that three CTAs fit on an SM next to their registers.
//
// dstate > 16: one CTA per (32 channels, group of 16 states), as in the forward.  Every state's
// reverse recurrence, its dA and its dB / dC rows belong to one CTA, but (S1, S2) sum over all
// states: with kMulti each CTA adds its partial pair per element into an fp32 workspace
// ([b][c][t][2]) and bwd_finish_kernel then forms du, ddelta, dz, dD and ddelta_bias.
#pragma once
#include "ss_common.cuh"
#include "ss_fwd.cuh"  // widen_bc

namespace ssb {

// tiles in flight per CTA: 3 for 2-byte I/O; 2 for fp32 I/O, whose larger tiles would
// otherwise leave room for only two CTAs per SM
template <typename IT>
constexpr int kStagesBwd = sizeof(IT) == 4 ? 2 : 3;
constexpr int kS12Row = 66;    // floats per row of the packed (S1, S2) partials (64 + 2 pad)

// dB/dC fold block: 16 rows of 64 floats (32 lanes x float2).  The per-row float2 writes cover
// 256 contiguous bytes; in the reduction, lane l reads row l >> 1 with 16-byte loads.  With
// 2-byte I/O the rows are kFoldRow = 72 floats apart, which puts the 4 rows of a quarter warp on
// distinct bank groups (72 r mod 32 = 8 r): both sides are conflict-free with addresses of the
// form per-lane base + constant.  With 4-byte I/O (no room for the pad) the rows are packed and
// 16-byte unit q of row r is stored at q ^ (2 (r & 3)), conflict-free on both sides as well.
template <typename IT> constexpr int kFoldRow = sizeof(IT) == 2 ? 72 : 64;
template <typename IT> __device__ __forceinline__ int fold_off(int r, int unit) {
  return sizeof(IT) == 2 ? r * 72 + 4 * unit : r * 64 + 4 * (unit ^ (2 * (r & 3)));
}

template <typename IT, int kNW, bool kVarB, bool kVarC, bool kHasZ>
struct BwdSmem {
  static constexpr int NS = kSPW * kNW;
  alignas(128) IT u[kStagesBwd<IT>][kCh][kTile];
  alignas(128) IT d[kStagesBwd<IT>][kCh][kTile];
  alignas(128) IT g[kStagesBwd<IT>][kCh][kTile];
  alignas(128) IT z[kHasZ ? kStagesBwd<IT> : 1][kCh][kTile];
  alignas(128) IT y[kHasZ ? kStagesBwd<IT> : 1][kCh][kTile];
  alignas(128) IT Braw[kVarB ? kStagesBwd<IT> : 1][NS * kTile];  // TMA path: B / C have the I/O dtype
  alignas(128) IT Craw[kVarC ? kStagesBwd<IT> : 1][NS * kTile];
  alignas(128) float hck[kStagesBwd<IT>][NS][kCh];   // states at the tile start, [n][channel]
  alignas(16) float4 dt_s[kCh][kElemRow<IT>];
  alignas(16) float4 dtu_s[kCh][kElemRow<IT>];
  alignas(16) float4 dy_s[kCh][kElemRow<IT>];
  alignas(16) float4 sig_s[kCh][4];
  alignas(16) float4 gz_s[kHasZ ? kCh : 1][4];
  alignas(16) float B_s[kVarB ? kTile : 1][NS];
  float bc_pad[16];  // puts C_s rows on the other half of the banks from B_s rows
  alignas(16) float C_s[kVarC ? kTile : 1][NS];
  alignas(16) float s12_s[kNW][kTile][kS12Row];                        // (S1, S2) per channel
  alignas(16) float fold[(kVarB || kVarC) ? kNW : 1][16 * kFoldRow<IT>];  // 4 steps x 2 pairs x B|C
  // per-warp channel sums of the tile: row k = (2 * pair + h) * 2 + (B|C), step t stored at
  // t ^ (4 * (k >> 1)), which makes the fold's scattered writes conflict-free while every
  // aligned group of 4 steps stays contiguous for the 16-byte reads
  alignas(16) float fout[(kVarB || kVarC) ? kNW : 1][2 * kSPW][kTile];
  alignas(8) uint64_t full[kStagesBwd<IT>];
};

template <typename IT, int kNW, bool kVarB, bool kVarC, bool kHasZ, bool kTMA, bool kMulti = false, bool kBLD = false>
__global__ void __launch_bounds__(32 * kNW, 3) ss_bwd_kernel(const __grid_constant__ BwdK P) {
  static_assert(!kBLD || (kTMA && !kMulti), "(b, L, d) tiles come from tensor maps, dstate <= 16");
  constexpr int NT = 32 * kNW;
  constexpr int NS = kSPW * kNW;
  constexpr int S = kTile / kNW;
  constexpr bool kFold = kVarB || kVarC;
  using Sm = BwdSmem<IT, kNW, kVarB, kVarC, kHasZ>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Sm& sm = *reinterpret_cast<Sm*>(smem_raw);
  const ss_bwd_args& a = P.a;
  const ss_fwd_args& f = a.f;

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int chunk = blockIdx.x % P.nchunk;
  const int cta = blockIdx.x / P.nchunk;
  const int ctile = cta % P.nct;
  const int bsg = cta / P.nct;
  const int sg = bsg % P.nsg;            // state group: states n0 .. n0 + 15
  const int b = bsg / P.nsg;
  const int grp = ctile / P.tpg;
  const int cl0 = (ctile % P.tpg) * kCh;
  const int c0 = grp * P.dpg + cl0;
  const int nvalid = min(kCh, P.dpg - cl0);
  const int n0 = sg * NS;
  const int N = f.dstate, L = f.seqlen;
  const bool bc_f32 = f.bc_dtype == SS_F32;

  // ---- scan role: channel c0 + lane, states 4w .. 4w+3 as pairs (4w, 4w+1), (4w+2, 4w+3)
  const bool lane_ok = lane < nvalid;
  const int c = c0 + lane;
  float2 A2[2], Ad[2], Bc[2], Cc[2], dA2[2], e2[2], dBc[2], dCc[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    float av[2], bv[2], cv[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int n = n0 + kSPW * w + 2 * p + h;
      const bool ok = lane_ok && n < N;
      const int64_t ia = (int64_t)c * N + n;
      av[h] = ok ? f.A[ia] : 0.f;
      bv[h] = 0.f;
      cv[h] = 0.f;
      if (!kVarB && ok) bv[h] = bc_f32 ? ((const float*)f.B)[ia] : to_f<IT>(((const IT*)f.B)[ia]);
      if (!kVarC && ok) cv[h] = bc_f32 ? ((const float*)f.C)[ia] : to_f<IT>(((const IT*)f.C)[ia]);
    }
    Ad[p] = make_float2(av[0], av[1]);
    A2[p] = make_float2(av[0] * kLog2e, av[1] * kLog2e);
    Bc[p] = make_float2(bv[0], bv[1]);
    Cc[p] = make_float2(cv[0], cv[1]);
    dA2[p] = e2[p] = dBc[p] = dCc[p] = make_float2(0.f, 0.f);
  }
  // ---- element role
  const int pc = elem_pc<kNW, kBLD>(tid), pq = elem_pq<kNW, kBLD>(tid);
  const bool pc_ok = pc < nvalid;
  const float Dv = (f.D != nullptr && pc_ok) ? f.D[c0 + pc] : 0.f;
  const float bias = (f.delta_bias != nullptr && pc_ok) ? f.delta_bias[c0 + pc] : 0.f;
  float dD_acc = 0.f, db_acc = 0.f;

  const IT* ub = (const IT*)f.u + (int64_t)b * f.u_batch_stride + (int64_t)c0 * f.u_dim_stride;
  const IT* db = (const IT*)f.delta + (int64_t)b * f.delta_batch_stride + (int64_t)c0 * f.delta_dim_stride;
  const IT* gb = (const IT*)a.dout + (int64_t)b * a.dout_batch_stride + (int64_t)c0 * a.dout_dim_stride;
  const IT* zb = kHasZ ? (const IT*)f.z + (int64_t)b * f.z_batch_stride + (int64_t)c0 * f.z_dim_stride : nullptr;
  const IT* yb = kHasZ ? (const IT*)a.y + (int64_t)b * a.y_batch_stride + (int64_t)c0 * a.y_dim_stride : nullptr;
  IT* du_row = (IT*)a.du + row_off<kBLD>(b, a.du_batch_stride, c0 + pc, a.du_dim_stride);
  IT* dd_row = (IT*)a.ddelta + row_off<kBLD>(b, a.ddelta_batch_stride, c0 + pc, a.ddelta_dim_stride);
  IT* dz_row = kHasZ ? (IT*)a.dz + row_off<kBLD>(b, a.dz_batch_stride, c0 + pc, a.dz_dim_stride) : nullptr;
  const int64_t bc_off = (((int64_t)b * f.ngroups + grp) * N + n0) * (int64_t)L;  // row n0 of this group

  const int ntiles = P.ntiles;
  const int kb = chunk * P.chunk_tiles;              // this CTA's tiles: kb .. kb + nt - 1
  const int nt = min(ntiles, kb + P.chunk_tiles) - kb;
  const uint32_t io_bytes = kCh * kTile * (uint32_t)sizeof(IT);
  const uint32_t bc_bytes = NS * kTile * (uint32_t)sizeof(IT);
  const uint32_t h_bytes = NS * kCh * 4u;
  // local iteration i handles tile kb + nt - 1 - i
  auto issue = [&](int i, int s) {
    const int k = kb + nt - 1 - i;
    uint64_t* bar = &sm.full[s];
    const uint32_t bytes = (3 + (kHasZ ? (kMulti ? 1 : 2) : 0)) * io_bytes +
                           ((kVarB ? 1 : 0) + (kVarC ? 1 : 0)) * bc_bytes + (k > 0 ? h_bytes : 0u);
    mbar_expect_tx(bar, bytes);
    const int t0 = k * kTile;
    const int x = kBLD ? c0 : t0, y = kBLD ? t0 : c0;  // (b, L, d) maps run along the channels
    tma_load_3d(&sm.u[s][0][0], &P.tm_u, x, y, b, bar);
    tma_load_3d(&sm.d[s][0][0], &P.tm_d, x, y, b, bar);
    tma_load_3d(&sm.g[s][0][0], &P.tm_g, x, y, b, bar);
    if constexpr (kHasZ) {
      tma_load_3d(&sm.z[s][0][0], &P.tm_z, x, y, b, bar);
      if constexpr (!kMulti) tma_load_3d(&sm.y[s][0][0], &P.tm_y, x, y, b, bar);
    }
    if constexpr (kVarB) tma_load_3d(&sm.Braw[s][0], &P.tm_B, t0, n0, b * f.ngroups + grp, bar);
    if constexpr (kVarC) tma_load_3d(&sm.Craw[s][0], &P.tm_C, t0, n0, b * f.ngroups + grp, bar);
    if (k > 0) tma_load_3d(&sm.hck[s][0][0], &P.tm_h, c0, n0, b * ntiles + (k - 1), bar);
  };
  if constexpr (kTMA) {
    if (tid == 0) {
      for (int s = 0; s < kStagesBwd<IT>; ++s) mbar_init(&sm.full[s], 1);
      mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0)
      for (int s = 0; s < kStagesBwd<IT> && s < nt; ++s) issue(s, s);
  }

  // a time chunk before the last starts from the carry the later chunks send back: chunk j
  // maps an incoming carry E to exp(A sum_j delta') E + (its local carry), folded over the
  // chunks after this one, last first.  The carries come from ss_bwd_carry_kernel, which this
  // launch may overlap (programmatic dependent launch): CTAs that read them wait for it here,
  // with their first tiles in flight.  A whole-row launch (zero_dep) waits here for the kernel
  // that zeroes the summed gradients before any of its atomic adds.
  if (chunk < P.nchunk - 1 || P.zero_dep) griddep_wait();
  if (chunk < P.nchunk - 1 && lane_ok) {
    for (int j = P.nchunk - 1; j > chunk; --j) {
      const int64_t bj = (int64_t)b * P.nchunk + j;
      const float sdt = P.csum[bj * f.dim + c];
      const float* cc = P.ccarry + (bj * N + kSPW * w) * (int64_t)f.dim + c;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const bool ok0 = kSPW * w + 2 * p < N, ok1 = kSPW * w + 2 * p + 1 < N;
        const float e0 = ok0 ? cc[(int64_t)(2 * p) * f.dim] : 0.f;
        const float e1 = ok1 ? cc[(int64_t)(2 * p + 1) * f.dim] : 0.f;
        e2[p].x = fmaf(ex2(A2[p].x * sdt), e2[p].x, e0);
        e2[p].y = fmaf(ex2(A2[p].y * sdt), e2[p].y, e1);
      }
    }
  }

  for (int it = 0; it < nt; ++it) {
    const int k = kb + nt - 1 - it;
    const int t0 = k * kTile;
    const int tlen = min(kTile, L - t0);
    const int stg = kTMA ? it % kStagesBwd<IT> : 0;
    bool failed = false;
    float2 hp[kTile + 1][2];
    if constexpr (kTMA) {
      failed = !mbar_wait_bounded(&sm.full[stg], (it / kStagesBwd<IT>) & 1, P.wait_cycles);
      if (w == 0) widen_bc_warp<IT, NS, kVarB, kVarC>(sm.B_s, sm.C_s, sm.Braw[stg], sm.Craw[stg], false, lane);
#pragma unroll
      for (int p = 0; p < 2; ++p)
        hp[0][p] = (k > 0) ? make_float2(sm.hck[stg][kSPW * w + 2 * p][lane], sm.hck[stg][kSPW * w + 2 * p + 1][lane])
                           : make_float2(0.f, 0.f);
    } else {
      load_tile<IT, NT>(sm.u[0], ub + t0, f.u_dim_stride, nvalid, tlen, P.vec_u);
      load_tile<IT, NT>(sm.d[0], db + t0, f.delta_dim_stride, nvalid, tlen, P.vec_d);
      load_tile<IT, NT>(sm.g[0], gb + t0, a.dout_dim_stride, nvalid, tlen, P.vec_dout);
      if constexpr (kHasZ) {
        load_tile<IT, NT>(sm.z[0], zb + t0, f.z_dim_stride, nvalid, tlen, P.vec_z);
        if constexpr (!kMulti) load_tile<IT, NT>(sm.y[0], yb + t0, a.y_dim_stride, nvalid, tlen, P.vec_y);
      }
      if constexpr (kVarB) {
        if (bc_f32) load_bc_tile<float, NT, NS>(sm.B_s, (const float*)f.B + bc_off + t0, L, N - n0, tlen);
        else load_bc_tile<IT, NT, NS>(sm.B_s, (const IT*)f.B + bc_off + t0, L, N - n0, tlen);
      }
      if constexpr (kVarC) {
        if (bc_f32) load_bc_tile<float, NT, NS>(sm.C_s, (const float*)f.C + bc_off + t0, L, N - n0, tlen);
        else load_bc_tile<IT, NT, NS>(sm.C_s, (const IT*)f.C + bc_off + t0, L, N - n0, tlen);
      }
      // states at the tile start (end of the previous tile), from the forward's checkpoints
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        float hv[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int n = n0 + kSPW * w + 2 * p + h;
          hv[h] = (k > 0 && lane_ok && n < N) ? f.ckpt[(((int64_t)b * ntiles + (k - 1)) * N + n) * f.dim + c] : 0.f;
        }
        hp[0][p] = make_float2(hv[0], hv[1]);
      }
      __syncthreads();
    }

    // ---- element phase 1: delta', delta'u, dy, softplus slope, gate slope
    {
      float uv[S], dv[S], gv[S], zv[S];
      lds_elems<IT, S, kBLD>(&sm.u[stg][0][0], pc, pq, uv);
      lds_elems<IT, S, kBLD>(&sm.d[stg][0][0], pc, pq, dv);
      lds_elems<IT, S, kBLD>(&sm.g[stg][0][0], pc, pq, gv);
      if constexpr (kHasZ) lds_elems<IT, S, kBLD>(&sm.z[stg][0][0], pc, pq, zv);
      float dtv[S], dtuv[S], dyv[S], sgv[S], gzv[S];
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const int t = pq * S + i;
        const bool ok = pc_ok && t < tlen;
        const float v = dv[i] + bias;
        float dt = v, sg = 1.f;
        if (f.delta_softplus) softplus_and_slope(v, dt, sg);
        float dy = gv[i], gz = 0.f;
        if constexpr (kHasZ) {
          const float sz = sigmoid_fast(zv[i]);
          dy = gv[i] * zv[i] * sz;
          gz = gv[i] * sz * fmaf(zv[i], 1.f - sz, 1.f);
        }
        if (!ok) {
          dt = 0.f;
          dy = 0.f;
        }
        dD_acc = fmaf(dy, uv[i], dD_acc);
        dtv[i] = dt;
        dtuv[i] = dt * uv[i];
        dyv[i] = dy;
        sgv[i] = sg;
        gzv[i] = gz;
      }
#pragma unroll
      for (int q = 0; q < S / 4; ++q) {
        const int ch = pq * (S / 4) + q;
        sm.dt_s[pc][erow<IT>(pc, ch)] = make_float4(dtv[4 * q], dtv[4 * q + 1], dtv[4 * q + 2], dtv[4 * q + 3]);
        sm.dtu_s[pc][erow<IT>(pc, ch)] = make_float4(dtuv[4 * q], dtuv[4 * q + 1], dtuv[4 * q + 2], dtuv[4 * q + 3]);
        sm.dy_s[pc][erow<IT>(pc, ch)] = make_float4(dyv[4 * q], dyv[4 * q + 1], dyv[4 * q + 2], dyv[4 * q + 3]);
        sm.sig_s[pc][ch] = make_float4(sgv[4 * q], sgv[4 * q + 1], sgv[4 * q + 2], sgv[4 * q + 3]);
        if constexpr (kHasZ)
          sm.gz_s[pc][ch] = make_float4(gzv[4 * q], gzv[4 * q + 1], gzv[4 * q + 2], gzv[4 * q + 3]);
      }
    }
    if (__syncthreads_or(failed)) {
      // a TMA stage did not complete in time: report, let every copy in flight land (this
      // tile's included: tiles it .. it + kStagesBwd - 1 were issued), and leave
      if (tid == 0) {
        if (P.status != nullptr) atomicOr(P.status, kStatusTimeout);
        for (int j = it; j < nt && j < it + kStagesBwd<IT>; ++j)
          mbar_wait_bounded(&sm.full[j % kStagesBwd<IT>], (j / kStagesBwd<IT>) & 1, kWaitCycles);
      }
      __syncthreads();
      return;
    }

    // ---- scan phase, forward: the states of the tile in registers.  The decays are not
    //      kept (the reverse sweep recomputes them): MUFU has headroom, registers do not,
    //      and the freed registers let the scheduler hide the shared-memory latencies.  Each
    //      group of 4 steps issues its 16 decays first (ordered ex2), ahead of the chain.
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
      const float4 du4 = sm.dtu_s[lane][erow<IT>(lane, i4)];
      const float4 dt4 = sm.dt_s[lane][erow<IT>(lane, i4)];
      const float dus[4] = {du4.x, du4.y, du4.z, du4.w};
      const float dts[4] = {dt4.x, dt4.y, dt4.z, dt4.w};
      float2 dg[4][2];  // the group's decays, issued ahead of the chain that consumes them
#pragma unroll
      for (int st = 0; st < 4; ++st)
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const float2 x = mul2(f2(dts[st]), A2[p]);
          dg[st][p] = make_float2(ex2_ordered(x.x), ex2_ordered(x.y));
        }
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        const int t = 4 * i4 + st;
        float2 Bv[2];
        if constexpr (kVarB) {
          const float4 q = *reinterpret_cast<const float4*>(&sm.B_s[t][kSPW * w]);
          Bv[0] = make_float2(q.x, q.y);
          Bv[1] = make_float2(q.z, q.w);
        } else {
          Bv[0] = Bc[0];
          Bv[1] = Bc[1];
        }
#pragma unroll
        for (int p = 0; p < 2; ++p) hp[t + 1][p] = fma2(dg[st][p], hp[t][p], mul2(f2(dus[st]), Bv[p]));
      }
    }

    // ---- scan phase, reverse
    float* fold = kFold ? &sm.fold[w][0] : nullptr;
#pragma unroll
    for (int i4 = 3; i4 >= 0; --i4) {
      const float4 dt4 = sm.dt_s[lane][erow<IT>(lane, i4)];
      const float4 du4 = sm.dtu_s[lane][erow<IT>(lane, i4)];
      const float4 dy4 = sm.dy_s[lane][erow<IT>(lane, i4)];
      const float dts[4] = {dt4.x, dt4.y, dt4.z, dt4.w};
      const float dus[4] = {du4.x, du4.y, du4.z, du4.w};
      const float dys[4] = {dy4.x, dy4.y, dy4.z, dy4.w};
      float2 dg[4][2];  // the group's decays, issued ahead of the reverse steps
#pragma unroll
      for (int st = 3; st >= 0; --st)
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const float2 x = mul2(f2(dts[st]), A2[p]);
          dg[st][p] = make_float2(ex2_ordered(x.x), ex2_ordered(x.y));
        }
#pragma unroll
      for (int st = 3; st >= 0; --st) {
        const int t = 4 * i4 + st;
        float2 Bv[2], Cv[2];
        if constexpr (kVarB) {
          const float4 q = *reinterpret_cast<const float4*>(&sm.B_s[t][kSPW * w]);
          Bv[0] = make_float2(q.x, q.y);
          Bv[1] = make_float2(q.z, q.w);
        } else {
          Bv[0] = Bc[0];
          Bv[1] = Bc[1];
        }
        if constexpr (kVarC) {
          const float4 q = *reinterpret_cast<const float4*>(&sm.C_s[t][kSPW * w]);
          Cv[0] = make_float2(q.x, q.y);
          Cv[1] = make_float2(q.z, q.w);
        } else {
          Cv[0] = Cc[0];
          Cv[1] = Cc[1];
        }
        const float2 dy2 = f2(dys[st]), du2 = f2(dus[st]), dt2 = f2(dts[st]);
        float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const float2 dh = fma2(Cv[p], dy2, e2[p]);
          const float2 ee = mul2(dg[st][p], dh);
          const float2 g = mul2(ee, hp[t][p]);
          dA2[p] = fma2(dt2, g, dA2[p]);
          s1 = fma2(Ad[p], g, s1);
          s2 = fma2(Bv[p], dh, s2);
          const float2 vB = mul2(dh, du2);
          const float2 vC = mul2(dy2, hp[t + 1][p]);
          if constexpr (kVarB)
            *reinterpret_cast<float2*>(fold + fold_off<IT>((st * 2 + p) * 2 + 0, lane >> 1) + 2 * (lane & 1)) = vB;
          else dBc[p] = add2(dBc[p], vB);
          if constexpr (kVarC)
            *reinterpret_cast<float2*>(fold + fold_off<IT>((st * 2 + p) * 2 + 1, lane >> 1) + 2 * (lane & 1)) = vC;
          else dCc[p] = add2(dCc[p], vC);
          e2[p] = ee;
        }
        *reinterpret_cast<float2*>(&sm.s12_s[w][t][2 * lane]) = make_float2(s1.x + s1.y, s2.x + s2.y);
      }
      if constexpr (kFold) {
        // sum the warp's 32 channels: lane l owns row r = l >> 1 = (step, pair, B|C) and reads
        // the float2 pairs of lanes 2(2m + h), 2(2m + h) + 1 for m = 0..7 (h = l & 1)
        __syncwarp();
        const int r = lane >> 1, h = lane & 1;
        const int type = r & 1;
        float2 acc = make_float2(0.f, 0.f);
        if ((type == 0 && kVarB) || (type == 1 && kVarC)) {
          float2 part[4];
#pragma unroll
          for (int m = 0; m < 8; ++m) {
            const float4 q = *reinterpret_cast<const float4*>(fold + fold_off<IT>(r, 2 * m + h));
            const float2 s2q = add2(make_float2(q.x, q.y), make_float2(q.z, q.w));
            part[m & 3] = (m < 4) ? s2q : add2(part[m & 3], s2q);
          }
          acc = add2(add2(part[0], part[1]), add2(part[2], part[3]));
        }
        acc.x += __shfl_xor_sync(0xffffffffu, acc.x, 1);
        acc.y += __shfl_xor_sync(0xffffffffu, acc.y, 1);
        const int st = r >> 2, p = (r >> 1) & 1;
        const int k = (2 * p + h) * 2 + type;
        sm.fout[w][k][(4 * i4 + st) ^ (4 * (k >> 1))] = h ? acc.y : acc.x;
        __syncwarp();
      }
    }

    // ---- dB / dC of this tile: 4 consecutive steps of one (B|C, n) row per lane
    if constexpr (kFold) {
      const int type = lane >> 4, j = (lane >> 2) & 3, tt = 4 * (lane & 3);
      const int n = kSPW * w + j;  // within the group: dst rows start at bc_off (row n0)
      const bool want = (type == 0) ? kVarB : kVarC;
      if (want && n0 + n < N) {
        const int k = j * 2 + type;
        const float4 v = *reinterpret_cast<const float4*>(&sm.fout[w][k][tt ^ (4 * (k >> 1))]);
        float* dst = (type == 0 ? a.dB : a.dC) + bc_off + (int64_t)n * L + t0 + tt;
        if (P.vec_dbc && tt + 4 <= tlen) {
          red_add_v4(dst, v.x, v.y, v.z, v.w);
        } else {
          const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (tt + i < tlen) red_add(dst + i, vv[i]);
        }
      }
    }
    // carry for the next (earlier) tile: e = exp(delta'_{t0} A) dh_{t0} is already in e2[]
    __syncthreads();

    // ---- element phase 2: du, ddelta, dz
    if constexpr (kMulti) {
      // state groups: this CTA's (S1, S2) over its states go to the workspace; the finish
      // kernel forms the element gradients from the sums over every group
      const int nv = pc_ok ? max(0, min(S, tlen - pq * S)) : 0;
      float* wrow = f.work + (((int64_t)b * f.dim + c0 + pc) * L + t0 + pq * S) * 2;
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const int t = pq * S + i;
        float2 S12 = make_float2(0.f, 0.f);
#pragma unroll
        for (int g = 0; g < kNW; ++g) S12 = add2(S12, *reinterpret_cast<const float2*>(&sm.s12_s[g][t][2 * pc]));
        if (i < nv) red_add_v2(wrow + 2 * i, S12.x, S12.y);
      }
    } else {
      float uv[S], yv[S];
      lds_elems<IT, S, kBLD>(&sm.u[stg][0][0], pc, pq, uv);
      if constexpr (kHasZ) lds_elems<IT, S, kBLD>(&sm.y[stg][0][0], pc, pq, yv);
      float duv[S], ddv[S], dzv[S];
#pragma unroll
      for (int q = 0; q < S / 4; ++q) {
        const int ch = pq * (S / 4) + q;
        const float4 dt4 = sm.dt_s[pc][erow<IT>(pc, ch)], dy4 = sm.dy_s[pc][erow<IT>(pc, ch)], sg4 = sm.sig_s[pc][ch];
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
          float2 S12 = make_float2(0.f, 0.f);
#pragma unroll
          for (int g = 0; g < kNW; ++g) S12 = add2(S12, *reinterpret_cast<const float2*>(&sm.s12_s[g][t][2 * pc]));
          duv[i] = fmaf(Dv, dys[r], dts[r] * S12.y);
          const float dd = fmaf(uv[i], S12.y, S12.x) * sgs[r];
          ddv[i] = dd;
          if (pc_ok && t < tlen) db_acc += dd;
          if constexpr (kHasZ) dzv[i] = gzs[r] * yv[i];
        }
      }
      const int nv = pc_ok ? max(0, min(S, tlen - pq * S)) : 0;
      store_elems<IT, S, kBLD>(du_row, step_stride<kBLD>(a.du_dim_stride), t0 + pq * S, duv, nv, P.vec_du);
      store_elems<IT, S, kBLD>(dd_row, step_stride<kBLD>(a.ddelta_dim_stride), t0 + pq * S, ddv, nv, P.vec_dd);
      if constexpr (kHasZ)
        store_elems<IT, S, kBLD>(dz_row, step_stride<kBLD>(a.dz_dim_stride), t0 + pq * S, dzv, nv, P.vec_dz);
    }
    __syncthreads();
    if constexpr (kTMA) {
      if (tid == 0 && it + kStagesBwd<IT> < nt) issue(it + kStagesBwd<IT>, stg);
    }
  }

  // ---- per-channel parameter gradients (summed over batch rows by the atomics)
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const float dAv[2] = {dA2[p].x, dA2[p].y}, dBv[2] = {dBc[p].x, dBc[p].y}, dCv[2] = {dCc[p].x, dCc[p].y};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int n = n0 + kSPW * w + 2 * p + h;
      if (lane_ok && n < N) {
        const int64_t ia = (int64_t)c * N + n;
        red_add(a.dA + ia, dAv[h]);
        if constexpr (!kVarB) red_add(a.dB + ia, dBv[h]);
        if constexpr (!kVarC) red_add(a.dC + ia, dCv[h]);
      }
    }
  }
  if constexpr (!kMulti) {  // (state groups: bwd_finish_kernel accumulates dD and ddelta_bias)
    if constexpr (!kBLD) {
      // the kNW element-role threads of a channel are adjacent lanes
#pragma unroll
      for (int o = 1; o < kNW; o <<= 1) {
        dD_acc += __shfl_xor_sync(0xffffffffu, dD_acc, o);
        db_acc += __shfl_xor_sync(0xffffffffu, db_acc, o);
      }
    }
    // ((b, L, d) tiles: the kNW threads of a channel sit in different warps and each adds its own)
    if ((kBLD || pq == 0) && pc_ok) {
      if (a.dD != nullptr) red_add(a.dD + c0 + pc, dD_acc);
      if (a.ddelta_bias != nullptr) red_add(a.ddelta_bias + c0 + pc, db_acc);
    }
  }
}

// dstate > 16: the element gradients from the (S1, S2) sums over every state group that the
// scan CTAs left in the workspace ([b][c][t][2]), with the element phases' formulas
// (backward_kernel.cu:499-521 and the gate):
//   du = D dy + delta' S2,   ddelta = (S1 + u S2) * softplus'(delta + bias),   dz = gz * y,
// plus dD += dy u and ddelta_bias += ddelta (one atomic per block: a block covers 256 steps of
// one (batch, channel) row).  One thread per element.
template <typename IT>
__global__ void __launch_bounds__(256) bwd_finish_kernel(const __grid_constant__ ss_bwd_args a, int nlc) {
  const ss_fwd_args& f = a.f;
  const int64_t row = blockIdx.x / nlc;               // b * dim + c
  const int t = (blockIdx.x % nlc) * 256 + threadIdx.x;
  const int64_t b = row / f.dim, c = row % f.dim;
  float dD = 0.f, db = 0.f;
  if (t < f.seqlen) {
    const float u = to_f<IT>(((const IT*)f.u)[b * f.u_batch_stride + c * f.u_dim_stride + t]);
    const float v = to_f<IT>(((const IT*)f.delta)[b * f.delta_batch_stride + c * f.delta_dim_stride + t]) +
                    (f.delta_bias != nullptr ? f.delta_bias[c] : 0.f);
    float dt = v, sg = 1.f;
    if (f.delta_softplus) softplus_and_slope(v, dt, sg);
    const float g = to_f<IT>(((const IT*)a.dout)[b * a.dout_batch_stride + c * a.dout_dim_stride + t]);
    float dy = g, gz = 0.f;
    if (f.z != nullptr) {
      const float zv = to_f<IT>(((const IT*)f.z)[b * f.z_batch_stride + c * f.z_dim_stride + t]);
      const float sz = sigmoid_fast(zv);
      dy = g * zv * sz;
      gz = g * sz * fmaf(zv, 1.f - sz, 1.f);
    }
    const float2 S12 = *reinterpret_cast<const float2*>(f.work + (row * f.seqlen + t) * 2);
    const float Dv = f.D != nullptr ? f.D[c] : 0.f;
    const float dd = fmaf(u, S12.y, S12.x) * sg;
    ((IT*)a.du)[b * a.du_batch_stride + c * a.du_dim_stride + t] = from_f<IT>(fmaf(Dv, dy, dt * S12.y));
    ((IT*)a.ddelta)[b * a.ddelta_batch_stride + c * a.ddelta_dim_stride + t] = from_f<IT>(dd);
    if (f.z != nullptr) {
      const float yv = to_f<IT>(((const IT*)a.y)[b * a.y_batch_stride + c * a.y_dim_stride + t]);
      ((IT*)a.dz)[b * a.dz_batch_stride + c * a.dz_dim_stride + t] = from_f<IT>(gz * yv);
    }
    dD = dy * u;
    db = dd;
  }
  __shared__ float red[2][8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    dD += __shfl_xor_sync(0xffffffffu, dD, o);
    db += __shfl_xor_sync(0xffffffffu, db, o);
  }
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
  if (lane == 0) {
    red[0][wid] = dD;
    red[1][wid] = db;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float sD = 0.f, sb = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      sD += red[0][i];
      sb += red[1][i];
    }
    if (a.dD != nullptr) red_add(a.dD + c, sD);
    if (a.ddelta_bias != nullptr) red_add(a.ddelta_bias + c, sb);
  }
}

}  // namespace ssb
