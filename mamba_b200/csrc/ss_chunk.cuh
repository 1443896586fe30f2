// Time-chunk passes of the selective scan (dstate <= 16, TMA path).
//
// The scan is sequential over time within a (batch, channel) row, so a grid of one CTA per
// (batch row, 32 channels) leaves most of the GPU idle when batch x dim is small (a batch of 1
// or 2 at d_inner 1536 - 5120 gives 48 - 160 CTAs for 148 SMs) however long the sequence is.
// Both recurrences are linear in their carried quantity, so the sequence can be cut into
// chunks that run in parallel once each chunk knows what enters it:
//
//   forward   H_out = exp(A * sum_chunk delta') H_in + s_chunk,   s_chunk = the chunk's end
//             state when it starts from zero (h_t = exp(delta'_t A) h_{t-1} + delta'_t u_t B_t);
//   backward  E_out = exp(A * sum_chunk delta') E_in + e_chunk,   e_chunk = the carry the
//             reverse recurrence (dh_t = C_t dy_t + E,  E <- exp(delta'_t A) dh_t) leaves at
//             the chunk's first step when it starts from zero at its last.
//
// ss_fwd_chunk_kernel computes (s_chunk, sum delta') for every chunk but the last, and
// ss_bwd_carry_kernel (e_chunk, sum delta') for every chunk but the first.  They are the
// recurrences alone — no outputs, no C.h in the forward, no states or gradients in the
// backward — so they cost a fraction of a full pass.  The main kernels then fold these
// summaries over the chunks before (forward) or after (backward) their own into their start
// state or carry, and run their chunk exactly as the unchunked kernel runs the whole row.
// The main kernels are launched as programmatic dependents of these passes: they start while a
// summary pass still runs, and only their CTAs that read summaries wait for it (the first chunk
// of the forward and the last chunk of the backward need none).
// This is the reference's per-chunk carry (forward_kernel.cu:274-286: the running prefix of
// (exp(delta' A), state) pairs across 2048-step chunks inside one CTA) spread over CTAs.
#pragma once
#include "ss_common.cuh"
#include "ss_fwd.cuh"  // widen_bc_warp

namespace ssb {

constexpr int kChunkStages = 4;

template <typename IT, int kNW, bool kVarB>
struct FwdChunkSmem {
  static constexpr int NS = kSPW * kNW;
  alignas(128) IT u[kChunkStages][kCh][kTile];
  alignas(128) IT d[kChunkStages][kCh][kTile];
  alignas(128) float Braw[kVarB ? kChunkStages : 1][NS * kTile];
  alignas(16) float4 dt_s[kCh][kElemRow<IT>];
  alignas(16) float4 dtu_s[kCh][kElemRow<IT>];
  alignas(16) float B_s[kVarB ? kTile : 1][NS];
  float part[kNW][kCh];  // per-warp partial sums of delta' ((b, L, d) tiles)
  alignas(8) uint64_t full[kChunkStages];
};

// Sum over the kNW element-role threads of channel pc of a per-thread partial, written by one of
// them to dst[pc] (pc < nvalid).  [channel][step] tiles: the threads are adjacent lanes (shuffles);
// [step][channel] tiles: they are lane pc of every warp (through shared memory).
template <int kNW, bool kBLD>
__device__ __forceinline__ void store_channel_sum(float v, float (*part)[kCh], float* dst, int pc, int pq, int nvalid) {
  if constexpr (kBLD) {
    part[pq][pc] = v;
    __syncthreads();
    if (pq == 0 && pc < nvalid) {
      float sum = 0.f;
#pragma unroll
      for (int g = 0; g < kNW; ++g) sum += part[g][pc];
      dst[pc] = sum;
    }
  } else {
#pragma unroll
    for (int o = 1; o < kNW; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (pq == 0 && pc < nvalid) dst[pc] = v;
  }
}

// Bounded wait for ring slot `stg`; on a timeout every thread learns of it, thread 0 raises the
// status bit and waits (with the default limit) for the copies of local tiles i .. issued - 1,
// and the caller returns.
__device__ __forceinline__ bool chunk_wait_failed(uint64_t* full, int stg, int i, int nt, int stages,
                                                  long long limit, int* status) {
  const bool failed = !mbar_wait_bounded(&full[stg], (i / stages) & 1, limit);
  if (__syncthreads_or(failed)) {
    if (threadIdx.x == 0) {
      if (status != nullptr) atomicOr(status, kStatusTimeout);
      for (int j = i; j < nt && j < i + stages; ++j) mbar_wait_bounded(&full[j % stages], (j / stages) & 1, kWaitCycles);
    }
    __syncthreads();
    return true;
  }
  return false;
}

// Forward chunk summaries: grid = batch x channel tiles x (nchunk - 1); CTA = (32 channels,
// chunk j < nchunk - 1), lane = channel, warp w = states 4w .. 4w+3 (as ss_fwd_kernel).
template <typename IT, int kNW, bool kVarB, bool kBLD>
__global__ void __launch_bounds__(32 * kNW, 4) ss_fwd_chunk_kernel(const __grid_constant__ FwdK P) {
  constexpr int NS = kSPW * kNW;
  constexpr int S = kTile / kNW;
  using Sm = FwdChunkSmem<IT, kNW, kVarB>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Sm& sm = *reinterpret_cast<Sm*>(smem_raw);
  const ss_fwd_args& a = P.a;

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int nch = P.nchunk - 1;
  const int chunk = blockIdx.x % nch;
  const int cta = blockIdx.x / nch;
  const int ctile = cta % P.nct;
  const int b = cta / P.nct;
  const int grp = ctile / P.tpg;
  const int cl0 = (ctile % P.tpg) * kCh;
  const int c0 = grp * P.dpg + cl0;
  const int nvalid = min(kCh, P.dpg - cl0);
  const int N = a.dstate, L = a.seqlen;
  const bool bc_f32 = a.bc_dtype == SS_F32;
  const int kb = chunk * P.chunk_tiles;
  const int nt = min(P.ntiles, kb + P.chunk_tiles) - kb;

  const bool lane_ok = lane < nvalid;
  const int c = c0 + lane;
  float2 A2[2], Bc[2], h[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    float av[2], bv[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int n = kSPW * w + 2 * p + q;
      const bool ok = lane_ok && n < N;
      const int64_t ia = (int64_t)c * N + n;
      av[q] = ok ? a.A[ia] * kLog2e : 0.f;
      bv[q] = 0.f;
      if (!kVarB && ok) bv[q] = bc_f32 ? ((const float*)a.B)[ia] : to_f<IT>(((const IT*)a.B)[ia]);
    }
    A2[p] = make_float2(av[0], av[1]);
    Bc[p] = make_float2(bv[0], bv[1]);
    h[p] = make_float2(0.f, 0.f);
  }
  const int pc = elem_pc<kNW, kBLD>(tid), pq = elem_pq<kNW, kBLD>(tid);
  const bool pc_ok = pc < nvalid;
  const float bias = (a.delta_bias != nullptr && pc_ok) ? a.delta_bias[c0 + pc] : 0.f;
  float dt_sum = 0.f;

  const uint32_t stage_bytes = 2 * kCh * kTile * (uint32_t)sizeof(IT) +
                               (kVarB ? NS * kTile * (bc_f32 ? 4u : (uint32_t)sizeof(IT)) : 0u);
  auto issue = [&](int i, int s) {
    uint64_t* bar = &sm.full[s];
    mbar_expect_tx(bar, stage_bytes);
    const int t0 = (kb + i) * kTile;
    const int x = kBLD ? c0 : t0, y = kBLD ? t0 : c0;  // (b, L, d) maps run along the channels
    tma_load_3d(&sm.u[s][0][0], &P.tm_u, x, y, b, bar);
    tma_load_3d(&sm.d[s][0][0], &P.tm_d, x, y, b, bar);
    if constexpr (kVarB) tma_load_3d(&sm.Braw[s][0], &P.tm_B, t0, 0, b * a.ngroups + grp, bar);
  };
  if (tid == 0) {
    for (int s = 0; s < kChunkStages; ++s) mbar_init(&sm.full[s], 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (tid == 0)
    for (int s = 0; s < kChunkStages && s < nt; ++s) issue(s, s);

  for (int i = 0; i < nt; ++i) {
    const int t0 = (kb + i) * kTile;
    const int tlen = min(kTile, L - t0);
    const int stg = i % kChunkStages;
    if (chunk_wait_failed(sm.full, stg, i, nt, kChunkStages, P.wait_cycles, P.status)) return;
    if (w == 0) widen_bc_warp<IT, NS, kVarB, false>(sm.B_s, sm.B_s, sm.Braw[stg], sm.Braw[stg], bc_f32, lane);
    {
      float uv[S], dv[S], dtv[S], dtuv[S];
      lds_elems<IT, S, kBLD>(&sm.u[stg][0][0], pc, pq, uv);
      lds_elems<IT, S, kBLD>(&sm.d[stg][0][0], pc, pq, dv);
#pragma unroll
      for (int k = 0; k < S; ++k) {
        const bool ok = pc_ok && pq * S + k < tlen;
        const float v = dv[k] + bias;
        float dt = a.delta_softplus ? softplus_thr(v) : v;
        dt = ok ? dt : 0.f;
        dt_sum += dt;
        dtv[k] = dt;
        dtuv[k] = dt * uv[k];
      }
#pragma unroll
      for (int q = 0; q < S / 4; ++q) {
        const int ch = pq * (S / 4) + q;
        sm.dt_s[pc][erow<IT>(pc, ch)] = make_float4(dtv[4 * q], dtv[4 * q + 1], dtv[4 * q + 2], dtv[4 * q + 3]);
        sm.dtu_s[pc][erow<IT>(pc, ch)] = make_float4(dtuv[4 * q], dtuv[4 * q + 1], dtuv[4 * q + 2], dtuv[4 * q + 3]);
      }
    }
    __syncthreads();
    // every thread is done with slot stg: refill it with the tile kChunkStages ahead
    if (tid == 0 && i + kChunkStages < nt) issue(i + kChunkStages, stg);
#pragma unroll
    for (int i4 = 0; i4 < 4; ++i4) {
      const float4 dt4 = sm.dt_s[lane][erow<IT>(lane, i4)];
      const float4 du4 = sm.dtu_s[lane][erow<IT>(lane, i4)];
      const float dts[4] = {dt4.x, dt4.y, dt4.z, dt4.w};
      const float dus[4] = {du4.x, du4.y, du4.z, du4.w};
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
        for (int p = 0; p < 2; ++p) {
          const float2 x = mul2(f2(dts[st]), A2[p]);
          h[p] = fma2(make_float2(ex2(x.x), ex2(x.y)), h[p], mul2(f2(dus[st]), Bv[p]));
        }
      }
    }
    __syncthreads();  // dt_s / dtu_s / B_s are rewritten by the next tile
  }

  // the main pass may start now (its CTAs that read the summaries wait for this grid to end)
  griddep_launch_dependents();
  const int64_t bj = (int64_t)b * P.nchunk + chunk;
  if (lane_ok) {
    const float hv[kSPW] = {h[0].x, h[0].y, h[1].x, h[1].y};
    float* cs = P.cstate + (bj * N) * (int64_t)a.dim + c;
#pragma unroll
    for (int j = 0; j < kSPW; ++j) {
      const int n = kSPW * w + j;
      if (n < N) cs[(int64_t)n * a.dim] = hv[j];
    }
  }
  store_channel_sum<kNW, kBLD>(dt_sum, sm.part, P.csum + bj * a.dim + c0, pc, pq, nvalid);
}

template <typename IT, int kNW, bool kVarC, bool kHasZ>
struct BwdCarrySmem {
  static constexpr int NS = kSPW * kNW;
  alignas(128) IT d[kChunkStages][kCh][kTile];
  alignas(128) IT g[kChunkStages][kCh][kTile];
  alignas(128) IT z[kHasZ ? kChunkStages : 1][kCh][kTile];
  alignas(128) IT Craw[kVarC ? kChunkStages : 1][NS * kTile];
  alignas(16) float4 dt_s[kCh][kElemRow<IT>];
  alignas(16) float4 dy_s[kCh][kElemRow<IT>];
  alignas(16) float C_s[kVarC ? kTile : 1][NS];
  float part[kNW][kCh];
  alignas(8) uint64_t full[kChunkStages];
};

// Backward chunk summaries: grid = batch x channel tiles x (nchunk - 1); CTA = (32 channels,
// chunk j >= 1), tiles visited last to first as in ss_bwd_kernel.
template <typename IT, int kNW, bool kVarC, bool kHasZ, bool kBLD>
__global__ void __launch_bounds__(32 * kNW, 4) ss_bwd_carry_kernel(const __grid_constant__ BwdK P) {
  constexpr int NS = kSPW * kNW;
  constexpr int S = kTile / kNW;
  using Sm = BwdCarrySmem<IT, kNW, kVarC, kHasZ>;
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Sm& sm = *reinterpret_cast<Sm*>(smem_raw);
  const ss_bwd_args& a = P.a;
  const ss_fwd_args& f = a.f;

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int nch = P.nchunk - 1;
  const int chunk = 1 + blockIdx.x % nch;
  const int cta = blockIdx.x / nch;
  const int ctile = cta % P.nct;
  const int b = cta / P.nct;
  const int grp = ctile / P.tpg;
  const int cl0 = (ctile % P.tpg) * kCh;
  const int c0 = grp * P.dpg + cl0;
  const int nvalid = min(kCh, P.dpg - cl0);
  const int N = f.dstate, L = f.seqlen;
  const bool bc_f32 = f.bc_dtype == SS_F32;
  const int kb = chunk * P.chunk_tiles;
  const int nt = min(P.ntiles, kb + P.chunk_tiles) - kb;

  const bool lane_ok = lane < nvalid;
  const int c = c0 + lane;
  float2 A2[2], Cc[2], e2[2];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    float av[2], cv[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const int n = kSPW * w + 2 * p + q;
      const bool ok = lane_ok && n < N;
      const int64_t ia = (int64_t)c * N + n;
      av[q] = ok ? f.A[ia] * kLog2e : 0.f;
      cv[q] = 0.f;
      if (!kVarC && ok) cv[q] = bc_f32 ? ((const float*)f.C)[ia] : to_f<IT>(((const IT*)f.C)[ia]);
    }
    A2[p] = make_float2(av[0], av[1]);
    Cc[p] = make_float2(cv[0], cv[1]);
    e2[p] = make_float2(0.f, 0.f);
  }
  const int pc = elem_pc<kNW, kBLD>(tid), pq = elem_pq<kNW, kBLD>(tid);
  const bool pc_ok = pc < nvalid;
  const float bias = (f.delta_bias != nullptr && pc_ok) ? f.delta_bias[c0 + pc] : 0.f;
  float dt_sum = 0.f;

  const uint32_t io_bytes = kCh * kTile * (uint32_t)sizeof(IT);
  const uint32_t stage_bytes = (2 + (kHasZ ? 1 : 0)) * io_bytes + (kVarC ? NS * kTile * (uint32_t)sizeof(IT) : 0u);
  auto issue = [&](int i, int s) {  // local iteration i handles tile kb + nt - 1 - i
    uint64_t* bar = &sm.full[s];
    mbar_expect_tx(bar, stage_bytes);
    const int t0 = (kb + nt - 1 - i) * kTile;
    const int x = kBLD ? c0 : t0, y = kBLD ? t0 : c0;
    tma_load_3d(&sm.d[s][0][0], &P.tm_d, x, y, b, bar);
    tma_load_3d(&sm.g[s][0][0], &P.tm_g, x, y, b, bar);
    if constexpr (kHasZ) tma_load_3d(&sm.z[s][0][0], &P.tm_z, x, y, b, bar);
    if constexpr (kVarC) tma_load_3d(&sm.Craw[s][0], &P.tm_C, t0, 0, b * f.ngroups + grp, bar);
  };
  if (tid == 0) {
    for (int s = 0; s < kChunkStages; ++s) mbar_init(&sm.full[s], 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (tid == 0)
    for (int s = 0; s < kChunkStages && s < nt; ++s) issue(s, s);

  for (int i = 0; i < nt; ++i) {
    const int t0 = (kb + nt - 1 - i) * kTile;
    const int tlen = min(kTile, L - t0);
    const int stg = i % kChunkStages;
    if (chunk_wait_failed(sm.full, stg, i, nt, kChunkStages, P.wait_cycles, P.status)) return;
    if (w == 0) widen_bc_warp<IT, NS, false, kVarC>(sm.C_s, sm.C_s, sm.Craw[stg], sm.Craw[stg], false, lane);
    {
      float dv[S], gv[S], zv[S], dtv[S], dyv[S];
      lds_elems<IT, S, kBLD>(&sm.d[stg][0][0], pc, pq, dv);
      lds_elems<IT, S, kBLD>(&sm.g[stg][0][0], pc, pq, gv);
      if constexpr (kHasZ) lds_elems<IT, S, kBLD>(&sm.z[stg][0][0], pc, pq, zv);
#pragma unroll
      for (int k = 0; k < S; ++k) {
        const bool ok = pc_ok && pq * S + k < tlen;
        const float v = dv[k] + bias;
        float dt = f.delta_softplus ? softplus_thr(v) : v;
        float dy = gv[k];
        if constexpr (kHasZ) dy = gv[k] * zv[k] * sigmoid_fast(zv[k]);
        dt = ok ? dt : 0.f;
        dy = ok ? dy : 0.f;
        dt_sum += dt;
        dtv[k] = dt;
        dyv[k] = dy;
      }
#pragma unroll
      for (int q = 0; q < S / 4; ++q) {
        const int ch = pq * (S / 4) + q;
        sm.dt_s[pc][erow<IT>(pc, ch)] = make_float4(dtv[4 * q], dtv[4 * q + 1], dtv[4 * q + 2], dtv[4 * q + 3]);
        sm.dy_s[pc][erow<IT>(pc, ch)] = make_float4(dyv[4 * q], dyv[4 * q + 1], dyv[4 * q + 2], dyv[4 * q + 3]);
      }
    }
    __syncthreads();
    if (tid == 0 && i + kChunkStages < nt) issue(i + kChunkStages, stg);
#pragma unroll
    for (int i4 = 3; i4 >= 0; --i4) {
      const float4 dt4 = sm.dt_s[lane][erow<IT>(lane, i4)];
      const float4 dy4 = sm.dy_s[lane][erow<IT>(lane, i4)];
      const float dts[4] = {dt4.x, dt4.y, dt4.z, dt4.w};
      const float dys[4] = {dy4.x, dy4.y, dy4.z, dy4.w};
#pragma unroll
      for (int st = 3; st >= 0; --st) {
        const int t = 4 * i4 + st;
        float2 Cv[2];
        if constexpr (kVarC) {
          const float4 q = *reinterpret_cast<const float4*>(&sm.C_s[t][kSPW * w]);
          Cv[0] = make_float2(q.x, q.y);
          Cv[1] = make_float2(q.z, q.w);
        } else {
          Cv[0] = Cc[0];
          Cv[1] = Cc[1];
        }
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const float2 dh = fma2(Cv[p], f2(dys[st]), e2[p]);
          const float2 x = mul2(f2(dts[st]), A2[p]);
          e2[p] = mul2(make_float2(ex2(x.x), ex2(x.y)), dh);
        }
      }
    }
    __syncthreads();
  }

  // the main pass may start now (its CTAs that read the summaries wait for this grid to end)
  griddep_launch_dependents();
  const int64_t bj = (int64_t)b * P.nchunk + chunk;
  if (lane_ok) {
    const float ev[kSPW] = {e2[0].x, e2[0].y, e2[1].x, e2[1].y};
    float* cc = P.ccarry + (bj * N) * (int64_t)f.dim + c;
#pragma unroll
    for (int j = 0; j < kSPW; ++j) {
      const int n = kSPW * w + j;
      if (n < N) cc[(int64_t)n * f.dim] = ev[j];
    }
  }
  store_channel_sum<kNW, kBLD>(dt_sum, sm.part, P.csum + bj * f.dim + c0, pc, pq, nvalid);
}

}  // namespace ssb
