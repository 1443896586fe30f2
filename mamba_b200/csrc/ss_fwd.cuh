// Forward selective scan for sm_100a.
//
// Computes, per (batch b, channel c) row and state n (reference forward_kernel.cu:213-293):
//   delta'_t = softplus(delta_t + bias_c)  (threshold 20)        [or delta_t + bias_c]
//   h_t[n]   = exp(delta'_t * A[c,n]) * h_{t-1}[n] + delta'_t * u_t * B_t[n]
//   y_t      = D_c * u_t + sum_n C_t[n] * h_t[n]
//   out_t    = y_t * silu(z_t)   when z is given (modules/mamba_simple.py:143-146)
//
// CTA = (32 channels of one group, one batch row); lane = channel, warp w = states 4w..4w+3.
// Inputs stream through a ring of kStages tile buffers in shared memory filled by TMA
// (cp.async.bulk.tensor, one elected thread, completion on an mbarrier per stage), so
// several 16-step tiles are in flight while the current one is computed.  Per tile:
//   1. each element's delta' and delta'*u is computed once and stored as fp32; the B / C
//      tiles (shared by all 32 channels) are widened to fp32 in [t][n] order;
//   2. every lane advances its 4 states through the 16 steps in registers — one ex2, one
//      FMUL, two FFMA per (element, state); the partial sum over its 4 states of C*h goes
//      to shared memory;
//   3. the warps' partial sums are added, D*u and the gate applied, and the tile stored;
//   4. the freed ring slot is refilled with the tile kStages ahead.
// At each tile end the 4 states of every lane go to the checkpoint buffer
// ckpt[b][tile][n][c] (coalesced over channels); the last tile's entry is the final state.
// When a tensor cannot be described by a TMA map (unaligned pointer or stride) the same
// kernel loads each tile synchronously with vector or scalar loads instead (kTMA = false).
//
// dstate > 16 (the reference's kernels take up to 256): the states split into groups of 16,
// one CTA per (32 channels, state group), each running its states from zero exactly as above.
// The sum over states then spans CTAs, so with kMulti each CTA adds its partial
// sum_n C*h (group 0 also D*u) into an fp32 workspace row with vector reductions instead of
// finishing the output; fwd_finish_kernel applies the gate and stores out / out_y afterwards.
// The grid is flattened: blockIdx.x = (batch row * state groups + group) * channel tiles + tile,
// so batch is not bound by gridDim.y.
#pragma once
#include "ss_common.cuh"

namespace ssb {

template <typename IT, int kNW, bool kVarB, bool kVarC, bool kHasZ>
struct FwdSmem {
  static constexpr int NS = kSPW * kNW;
  alignas(128) IT u[kStages][kCh][kTile];
  alignas(128) IT d[kStages][kCh][kTile];
  alignas(128) IT z[kHasZ ? kStages : 1][kCh][kTile];
  alignas(128) float Braw[kVarB ? kStages : 1][NS * kTile];  // TMA tile of B (its own dtype)
  alignas(128) float Craw[kVarC ? kStages : 1][NS * kTile];
  alignas(16) float4 dt_s[kCh][kElemRow<IT>];
  alignas(16) float4 dtu_s[kCh][kElemRow<IT>];
  alignas(16) float B_s[kVarB ? kTile : 1][NS];
  float bc_pad[16];  // puts C_s rows on the other half of the banks from B_s rows
  alignas(16) float C_s[kVarC ? kTile : 1][NS];
  float y_s[2][kNW][kTile][kPad];  // per-warp partial outputs, double-buffered across tiles
  alignas(8) uint64_t full[kStages];
};

// B and C tiles arrive from TMA as raw[n][t] (NS rows of kTile steps, in the I/O dtype, or fp32
// when f32) and the scans read them as fp32 [t][n].  One warp transposes both: lane l < 16
// owns row l of B, lane l >= 16 row l - 16 of C; it reads its row with 16-byte loads and
// writes one column, so each store instruction covers 16 consecutive floats of a B row and 16
// of a C row (on different bank halves: C_s is laid out 16 floats off B_s's banks).  A
// thread-per-element mapping made every store an 8-way bank conflict.
template <typename IT, int NS, bool kB, bool kC>
__device__ __forceinline__ void widen_bc_warp(float (*Bd)[NS], float (*Cd)[NS], const void* Braw, const void* Craw,
                                              bool f32, int lane) {
  const bool isC = lane >= 16;
  const int n = lane & 15;
  if (n >= NS || (isC ? !kC : !kB)) return;
  float (*dst)[NS] = isC ? Cd : Bd;
  const void* raw = isC ? Craw : Braw;
  float v[kTile];
  if (f32) {
    const float4* r = reinterpret_cast<const float4*>(static_cast<const float*>(raw) + n * kTile);
#pragma unroll
    for (int q = 0; q < kTile / 4; ++q) {
      const float4 x = r[q];
      v[4 * q] = x.x; v[4 * q + 1] = x.y; v[4 * q + 2] = x.z; v[4 * q + 3] = x.w;
    }
  } else {
    constexpr int VW = 16 / sizeof(IT);
    const uint4* r = reinterpret_cast<const uint4*>(static_cast<const IT*>(raw) + n * kTile);
#pragma unroll
    for (int q = 0; q < kTile / VW; ++q) {
      const uint4 x = r[q];
      const IT* e = reinterpret_cast<const IT*>(&x);
#pragma unroll
      for (int j = 0; j < VW; ++j) v[q * VW + j] = to_f<IT>(e[j]);
    }
  }
#pragma unroll
  for (int t = 0; t < kTile; ++t) dst[t][n] = v[t];
}

template <typename IT, int kNW, bool kVarB, bool kVarC, bool kHasZ, bool kTMA, bool kMulti = false, bool kBLD = false>
__global__ void __launch_bounds__(32 * kNW, 4) ss_fwd_kernel(const __grid_constant__ FwdK P) {
  static_assert(!(kMulti && kHasZ), "state groups apply the gate in fwd_finish_kernel");
  static_assert(!kBLD || (kTMA && !kMulti), "(b, L, d) tiles come from tensor maps, dstate <= 16");
  constexpr int NT = 32 * kNW;
  constexpr int NS = kSPW * kNW;   // states covered by the CTA (dstate padded up)
  constexpr int S = kTile / kNW;   // steps per thread in the element-wise phases
  using Sm = FwdSmem<IT, kNW, kVarB, kVarC, kHasZ>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Sm& sm = *reinterpret_cast<Sm*>(smem_raw);
  const ss_fwd_args& a = P.a;

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
  const int n0 = sg * kSPW * kNW;
  const int N = a.dstate, L = a.seqlen;
  const bool bc_f32 = a.bc_dtype == SS_F32;
  const int ntiles = P.ntiles;
  const int kb = chunk * P.chunk_tiles;              // this CTA's tiles: kb .. kb + nt - 1
  const int nt = min(ntiles, kb + P.chunk_tiles) - kb;

  // ---- scan role: channel c0 + lane, states kSPW*w + j
  const bool lane_ok = lane < nvalid;
  const int c = c0 + lane;
  float2 A2[2], Bc[2], Cc[2], h[2];   // states (4w, 4w+1), (4w+2, 4w+3) as packed pairs
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    float av[2], bv[2], cv[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int n = n0 + kSPW * w + 2 * p + q;
      const bool ok = lane_ok && n < N;
      const int64_t ia = (int64_t)c * N + n;
      av[q] = ok ? a.A[ia] * kLog2e : 0.f;
      bv[q] = 0.f;
      cv[q] = 0.f;
      if (!kVarB && ok) bv[q] = bc_f32 ? ((const float*)a.B)[ia] : to_f<IT>(((const IT*)a.B)[ia]);
      if (!kVarC && ok) cv[q] = bc_f32 ? ((const float*)a.C)[ia] : to_f<IT>(((const IT*)a.C)[ia]);
    }
    A2[p] = make_float2(av[0], av[1]);
    Bc[p] = make_float2(bv[0], bv[1]);
    Cc[p] = make_float2(cv[0], cv[1]);
    h[p] = make_float2(0.f, 0.f);
  }
  // ---- element role: channel c0 + pc, steps pq*S .. pq*S + S - 1 of each tile
  const int pc = elem_pc<kNW, kBLD>(tid), pq = elem_pq<kNW, kBLD>(tid);
  const bool pc_ok = pc < nvalid;
  const float Dv = (a.D != nullptr && pc_ok) ? a.D[c0 + pc] : 0.f;
  const float bias = (a.delta_bias != nullptr && pc_ok) ? a.delta_bias[c0 + pc] : 0.f;
  IT* orow = (IT*)a.out + row_off<kBLD>(b, a.out_batch_stride, c0 + pc, a.out_dim_stride);
  const int64_t ostep = step_stride<kBLD>(a.out_dim_stride);
  IT* yrow = (kHasZ && a.out_y != nullptr)
                 ? (IT*)a.out_y + row_off<kBLD>(b, a.out_y_batch_stride, c0 + pc, a.out_y_dim_stride)
                 : nullptr;
  const int64_t ystep = step_stride<kBLD>(a.out_y_dim_stride);
  const int64_t bc_off = (((int64_t)b * a.ngroups + grp) * N + n0) * (int64_t)L;  // row n0 of this group

  // ---- producer (thread 0): TMA ring
  const uint32_t bc_bytes = NS * kTile * (bc_f32 ? 4u : (uint32_t)sizeof(IT));
  const uint32_t stage_bytes = (2 + (kHasZ ? 1 : 0)) * kCh * kTile * (uint32_t)sizeof(IT) +
                               ((kVarB ? 1 : 0) + (kVarC ? 1 : 0)) * bc_bytes;
  auto issue = [&](int i, int s) {  // local tile i (global tile kb + i) into ring slot s
    uint64_t* bar = &sm.full[s];
    mbar_expect_tx(bar, stage_bytes);
    const int t0 = (kb + i) * kTile;
    const int x = kBLD ? c0 : t0, y = kBLD ? t0 : c0;  // (b, L, d) maps run along the channels
    tma_load_3d(&sm.u[s][0][0], &P.tm_u, x, y, b, bar);
    tma_load_3d(&sm.d[s][0][0], &P.tm_d, x, y, b, bar);
    if constexpr (kHasZ) tma_load_3d(&sm.z[s][0][0], &P.tm_z, x, y, b, bar);
    if constexpr (kVarB) tma_load_3d(&sm.Braw[s][0], &P.tm_B, t0, n0, b * a.ngroups + grp, bar);
    if constexpr (kVarC) tma_load_3d(&sm.Craw[s][0], &P.tm_C, t0, n0, b * a.ngroups + grp, bar);
  };
  if constexpr (kTMA) {
    if (tid == 0) {
      for (int s = 0; s < kStages; ++s) mbar_init(&sm.full[s], 1);
      mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0)
      for (int s = 0; s < kStages && s < nt; ++s) issue(s, s);
  }

  const IT* ub = (const IT*)a.u + (int64_t)b * a.u_batch_stride + (int64_t)c0 * a.u_dim_stride;
  const IT* db = (const IT*)a.delta + (int64_t)b * a.delta_batch_stride + (int64_t)c0 * a.delta_dim_stride;
  const IT* zb = kHasZ ? (const IT*)a.z + (int64_t)b * a.z_batch_stride + (int64_t)c0 * a.z_dim_stride : nullptr;

  // a later time chunk starts from the state the earlier chunks leave behind: chunk j maps a
  // start state H to exp(A sum_j delta') H + (its local end state), folded over j < chunk.  The
  // summaries come from ss_fwd_chunk_kernel, which this launch may overlap (programmatic
  // dependent launch): CTAs that read them wait for it here, with their first tiles in flight.
  if (chunk > 0) griddep_wait();
  if (chunk > 0 && lane_ok) {
    for (int j = 0; j < chunk; ++j) {
      const int64_t bj = (int64_t)b * P.nchunk + j;
      const float sdt = P.csum[bj * a.dim + c];
      const float* cs = P.cstate + (bj * N + kSPW * w) * (int64_t)a.dim + c;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        const bool ok0 = kSPW * w + 2 * p < N, ok1 = kSPW * w + 2 * p + 1 < N;
        const float s0 = ok0 ? cs[(int64_t)(2 * p) * a.dim] : 0.f;
        const float s1 = ok1 ? cs[(int64_t)(2 * p + 1) * a.dim] : 0.f;
        h[p].x = fmaf(ex2(A2[p].x * sdt), h[p].x, s0);
        h[p].y = fmaf(ex2(A2[p].y * sdt), h[p].y, s1);
      }
    }
  }

  for (int it = 0; it < nt; ++it) {
    const int k = kb + it;  // global tile
    const int t0 = k * kTile;
    const int tlen = min(kTile, L - t0);
    const int stg = kTMA ? it % kStages : 0;
    const int yb = it & 1;  // y_s buffer of this tile
    bool failed = false;
    if constexpr (kTMA) {
      failed = !mbar_wait_bounded(&sm.full[stg], (it / kStages) & 1, P.wait_cycles);
      if (w == 0) widen_bc_warp<IT, NS, kVarB, kVarC>(sm.B_s, sm.C_s, sm.Braw[stg], sm.Craw[stg], bc_f32, lane);
    } else {
      load_tile<IT, NT>(sm.u[0], ub + t0, a.u_dim_stride, nvalid, tlen, P.vec_u);
      load_tile<IT, NT>(sm.d[0], db + t0, a.delta_dim_stride, nvalid, tlen, P.vec_d);
      if constexpr (kHasZ) load_tile<IT, NT>(sm.z[0], zb + t0, a.z_dim_stride, nvalid, tlen, P.vec_z);
      if constexpr (kVarB) {
        if (bc_f32) load_bc_tile<float, NT, NS>(sm.B_s, (const float*)a.B + bc_off + t0, L, N - n0, tlen);
        else load_bc_tile<IT, NT, NS>(sm.B_s, (const IT*)a.B + bc_off + t0, L, N - n0, tlen);
      }
      if constexpr (kVarC) {
        if (bc_f32) load_bc_tile<float, NT, NS>(sm.C_s, (const float*)a.C + bc_off + t0, L, N - n0, tlen);
        else load_bc_tile<IT, NT, NS>(sm.C_s, (const IT*)a.C + bc_off + t0, L, N - n0, tlen);
      }
      __syncthreads();
    }

    // ---- 1. delta' and delta'*u, once per element (steps past seqlen get delta' = 0,
    //         so the states pass through them unchanged)
    {
      float uv[S], dv[S], dtv[S], dtuv[S];
      lds_elems<IT, S, kBLD>(&sm.u[stg][0][0], pc, pq, uv);
      lds_elems<IT, S, kBLD>(&sm.d[stg][0][0], pc, pq, dv);
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const int t = pq * S + i;
        const bool ok = pc_ok && t < tlen;
        const float v = dv[i] + bias;
        float dt = a.delta_softplus ? softplus_thr(v) : v;
        dt = ok ? dt : 0.f;
        dtv[i] = dt;
        dtuv[i] = dt * uv[i];
      }
#pragma unroll
      for (int q = 0; q < S / 4; ++q) {
        const int ch = pq * (S / 4) + q;
        sm.dt_s[pc][erow<IT>(pc, ch)] = make_float4(dtv[4 * q], dtv[4 * q + 1], dtv[4 * q + 2], dtv[4 * q + 3]);
        sm.dtu_s[pc][erow<IT>(pc, ch)] = make_float4(dtuv[4 * q], dtuv[4 * q + 1], dtuv[4 * q + 2], dtuv[4 * q + 3]);
      }
    }
    if (__syncthreads_or(failed)) {  // (every thread has also finished the previous tile's epilogue)
      // a TMA stage did not complete in time: report, let every copy in flight land (this
      // tile's included), and leave
      if (tid == 0) {
        if (P.status != nullptr) atomicOr(P.status, kStatusTimeout);
        const int issued_end = max(kStages, it + kStages - 1);  // local tiles issued before this point
        for (int j = it; j < nt && j < issued_end; ++j)
          mbar_wait_bounded(&sm.full[j % kStages], (j / kStages) & 1, kWaitCycles);
      }
      __syncthreads();
      return;
    }
    // ---- refill the slot the previous tile used (every thread is past its epilogue)
    if constexpr (kTMA) {
      if (tid == 0 && it >= 1 && it - 1 + kStages < nt) issue(it - 1 + kStages, (it - 1) % kStages);
    }

    // ---- 2. the recurrence, 4 states per lane, 16 steps.  All 64 decays of the tile are
    //         issued first (independent ex2, so the MUFU pipe stays full), then the FMA
    //         recurrence consumes them.
    float2 da[kTile][2];
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
      const float4 dt4 = sm.dt_s[lane][erow<IT>(lane, i4)];
      const float dts[4] = {dt4.x, dt4.y, dt4.z, dt4.w};
#pragma unroll
      for (int st = 0; st < 4; ++st)
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const float2 x = mul2(f2(dts[st]), A2[p]);
          da[4 * i4 + st][p] = make_float2(ex2_ordered(x.x), ex2_ordered(x.y));
        }
    }
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
      const float4 du4 = sm.dtu_s[lane][erow<IT>(lane, i4)];
      const float dus[4] = {du4.x, du4.y, du4.z, du4.w};
#pragma unroll
      for (int st = 0; st < 4; ++st) {
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
#pragma unroll
        for (int p = 0; p < 2; ++p) h[p] = fma2(da[t][p], h[p], mul2(f2(dus[st]), Bv[p]));
        const float2 y2 = fma2(Cv[1], h[1], mul2(Cv[0], h[0]));
        sm.y_s[yb][w][t][lane] = y2.x + y2.y;
      }
    }
    if (a.ckpt != nullptr && lane_ok) {
      float* ck = a.ckpt + ((int64_t)b * ntiles + k) * N * (int64_t)a.dim + c;
      const float hv[kSPW] = {h[0].x, h[0].y, h[1].x, h[1].y};
#pragma unroll
      for (int j = 0; j < kSPW; ++j) {
        const int n = n0 + kSPW * w + j;
        if (n < N) ck[(int64_t)n * a.dim] = hv[j];
      }
    }
    __syncthreads();

    // ---- 3. combine the warps' partial sums, add D*u, gate, store
    if constexpr (kMulti) {
      // state groups: this CTA's share of y (group 0 adds D*u) goes to the fp32 workspace
      float uo[S], ys[S];
      lds_elems<IT, S, kBLD>(&sm.u[stg][0][0], pc, pq, uo);
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const int t = pq * S + i;
        float y = sg == 0 ? Dv * uo[i] : 0.f;
#pragma unroll
        for (int g = 0; g < kNW; ++g) y += sm.y_s[yb][g][t][pc];
        ys[i] = y;
      }
      const int nv = pc_ok ? max(0, min(S, tlen - pq * S)) : 0;
      float* wrow = a.work + ((int64_t)b * a.dim + c0 + pc) * L + t0 + pq * S;
      if (P.vec_work && nv == S) {
#pragma unroll
        for (int i = 0; i < S; i += 4) red_add_v4(wrow + i, ys[i], ys[i + 1], ys[i + 2], ys[i + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < S; ++i)
          if (i < nv) red_add(wrow + i, ys[i]);
      }
    } else {
      float yv[S], uo[S], zo[S], yu[S];
      lds_elems<IT, S, kBLD>(&sm.u[stg][0][0], pc, pq, uo);
      if constexpr (kHasZ) lds_elems<IT, S, kBLD>(&sm.z[stg][0][0], pc, pq, zo);
#pragma unroll
      for (int i = 0; i < S; ++i) {
        const int t = pq * S + i;
        float y = Dv * uo[i];
#pragma unroll
        for (int g = 0; g < kNW; ++g) y += sm.y_s[yb][g][t][pc];
        yu[i] = y;
        if constexpr (kHasZ) {
          y *= zo[i] * sigmoid_fast(zo[i]);
        }
        yv[i] = y;
      }
      const int nv = pc_ok ? max(0, min(S, tlen - pq * S)) : 0;
      store_elems<IT, S, kBLD>(orow, ostep, t0 + pq * S, yv, nv, P.vec_out);
      if (kHasZ && yrow != nullptr) store_elems<IT, S, kBLD>(yrow, ystep, t0 + pq * S, yu, nv, P.vec_y);
    }
    // With TMA there is no barrier here: the next tile's recurrence writes the other y_s buffer,
    // and the slot this epilogue read is refilled only after the next tile's first barrier,
    // which every thread reaches after finishing this epilogue.  The synchronous path reloads
    // its single slot at the top of the next tile, so it waits here.
    if constexpr (!kTMA) __syncthreads();
  }

  if (a.last_state != nullptr && lane_ok && chunk == P.nchunk - 1) {
    float* ls = a.last_state + ((int64_t)b * a.dim + c) * N;
    const float hv[kSPW] = {h[0].x, h[0].y, h[1].x, h[1].y};
#pragma unroll
    for (int j = 0; j < kSPW; ++j) {
      const int n = n0 + kSPW * w + j;
      if (n < N) ls[n] = hv[j];
    }
  }
}

// dstate > 16: out = work * silu(z) (or work), out_y = work when a gate is given; work holds
// D*u + sum over all states of C*h for every (batch, channel, step), packed [b][c][t].
// One thread per element; the grid is flattened over rows x 256-step chunks.
template <typename IT>
__global__ void __launch_bounds__(256) fwd_finish_kernel(const __grid_constant__ ss_fwd_args a, int nlc) {
  const int64_t row = blockIdx.x / nlc;              // b * dim + c
  const int t = (blockIdx.x % nlc) * 256 + threadIdx.x;
  if (t >= a.seqlen) return;
  const int64_t b = row / a.dim, c = row % a.dim;
  float y = a.work[row * a.seqlen + t];
  if (a.z != nullptr) {
    const float zv = to_f<IT>(((const IT*)a.z)[b * a.z_batch_stride + c * a.z_dim_stride + t]);
    if (a.out_y != nullptr) ((IT*)a.out_y)[b * a.out_y_batch_stride + c * a.out_y_dim_stride + t] = from_f<IT>(y);
    y *= zv * sigmoid_fast(zv);
  }
  ((IT*)a.out)[b * a.out_batch_stride + c * a.out_dim_stride + t] = from_f<IT>(y);
}

}  // namespace ssb
