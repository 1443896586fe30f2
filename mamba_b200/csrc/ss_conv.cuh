// Causal depthwise convolution + SiLU on the input side of a Mamba block, fused with the
// layout change the reference does with permute().contiguous() copies
// (modules/mamba_simple.py:91-98: input_proj -> permute -> chunk -> short_conv -> SiLU;
// the conv is nn.Conv1d(groups=dim, padding=width-1) truncated to seqlen, :41-48, :97):
//
//   pre[b,c,t] = bias[c] + sum_{k<K} w[c,k] * x[b, t-(K-1)+k, c]     (x[t<0] = state or 0)
//   u[b,c,t]   = silu(pre[b,c,t])
//
// x (and the gate half z) arrive in the input projection's (batch, seqlen, dim) layout,
// channels contiguous; u (and the transposed z) leave in the scan's (batch, dim, seqlen)
// layout.  One CTA of 256 threads owns a 64-step x 64-channel tile: it reads the tile's rows
// (plus the K-1 steps before it) with 16-byte loads along channels into shared memory, and
// each thread then produces 16 consecutive steps of one channel and writes them with 16-byte
// stores along the sequence, so both sides stay coalesced.  HBM-bound: per element it reads
// x (and z) and writes u (and zt) once.
//
// The backward recomputes pre from x, forms dpre = du * silu'(pre) for the tile and the K-1
// steps after it (in shared memory), and produces
//   dx[t]    = sum_k w[k] dpre[t+(K-1)-k]       (written back in the (batch, seqlen, dim) layout)
//   dw[c,k] += sum_t dpre[t] x[t-(K-1)+k],  dbias[c] += sum_t dpre[t]
// with the per-channel sums reduced over the CTA's threads before one atomic per channel
// and CTA.  The decode step applies the same window to one new input and rolls the state.
#pragma once
#include "ss_common.cuh"

namespace ssb {

constexpr int kConvT = 64;   // steps per tile
constexpr int kConvC = 64;   // channels per tile
constexpr int kConvThreads = 256;
constexpr int kConvTPT = 16; // steps per thread (kConvThreads / kConvC thread rows of 16)

// The conv grids are flattened: blockIdx.x = (batch row * nt + step tile) * nc + channel
// tile, so no size is bound by gridDim.y / gridDim.z.
struct ConvK {
  ss_conv_args a;
  int nc, nt;   // channel tiles, step tiles
  int vec_x;    // x rows 16-byte aligned with dim a multiple of the vector width
  int vec_u;    // u rows 16-byte aligned
  int vec_z, vec_zt;
};

struct ConvBwdK {
  ss_conv_bwd_args a;
  int nc, nt;
  int vec_x, vec_du, vec_dx, vec_dzt, vec_dz;
};

// Load rows of a (seqlen, dim) slab (row r is step t_first + r) for channels [c0, c0 + 64)
// into dst[row][64], keeping the I/O dtype: one 16-byte shared store per 16-byte global
// load, so a quarter-warp writes one contiguous 128-byte row segment (no bank conflicts).
// Rows before t = 0 come from state (b, dim, K-1, fp32) or are zero; rows at or past seqlen
// and channels past dim are zero.
template <typename IT, int K>
__device__ __forceinline__ void conv_load_rows(IT* dst, int nrows, const IT* xb, int64_t seq_stride, int t_first,
                                               int c0, int dim, int L, const float* state_b, bool vec) {
  constexpr int VW = 16 / sizeof(IT);  // elements per 16-byte vector
  constexpr int CH = kConvC / VW;      // vectors per row
  for (int i = threadIdx.x; i < nrows * CH; i += kConvThreads) {
    const int r = i / CH, ch = (i % CH) * VW;
    const int t = t_first + r;
    uint4 pk = make_uint4(0u, 0u, 0u, 0u);
    IT* e = reinterpret_cast<IT*>(&pk);
    if (t >= 0 && t < L) {
      const IT* src = xb + (int64_t)t * seq_stride + c0 + ch;
      if (vec && c0 + ch + VW <= dim) {
        pk = *reinterpret_cast<const uint4*>(src);
      } else {
#pragma unroll
        for (int j = 0; j < VW; ++j)
          if (c0 + ch + j < dim) e[j] = src[j];
      }
    } else if (t < 0 && t >= -(K - 1) && state_b != nullptr) {
#pragma unroll
      for (int j = 0; j < VW; ++j)
        if (c0 + ch + j < dim) e[j] = from_f<IT>(state_b[(int64_t)(c0 + ch + j) * (K - 1) + (t + K - 1)]);
    }
    *reinterpret_cast<uint4*>(dst + r * kConvC + ch) = pk;
  }
}

// Write rows of a [64 t][64 c] tile (I/O dtype) into a (seqlen, dim) slab: one 16-byte
// shared load and one 16-byte global store per vector.
template <typename IT>
__device__ __forceinline__ void conv_store_rows(IT* yb, int64_t seq_stride, const IT* src, int t0, int c0, int dim,
                                                int L, bool vec) {
  constexpr int VW = 16 / sizeof(IT);
  constexpr int CH = kConvC / VW;
  for (int i = threadIdx.x; i < kConvT * CH; i += kConvThreads) {
    const int r = i / CH, ch = (i % CH) * VW;
    const int t = t0 + r;
    if (t >= L) continue;
    IT* dst = yb + (int64_t)t * seq_stride + c0 + ch;
    const uint4 pk = *reinterpret_cast<const uint4*>(src + r * kConvC + ch);
    if (vec && c0 + ch + VW <= dim) {
      *reinterpret_cast<uint4*>(dst) = pk;
    } else {
      const IT* e = reinterpret_cast<const IT*>(&pk);
#pragma unroll
      for (int j = 0; j < VW; ++j)
        if (c0 + ch + j < dim) dst[j] = e[j];
    }
  }
}

// Row pitch (elements) of a [channel][step] staging tile: 64 steps plus one 16-byte vector
// of padding, so rows start 4 banks apart and the per-channel 16-byte accesses of a warp
// (one channel per lane) are conflict-free.  Also leaves room for the K-1 <= 3 halo steps.
template <typename IT>
constexpr int conv_pitch() { return kConvT + 16 / (int)sizeof(IT); }

// Load the [64 channels][ncols steps] block starting at (c0, t0) of a (dim, seqlen) slab
// (row stride dim_stride) into dst[c][conv_pitch] with row-contiguous 16-byte loads (8 or 16
// threads per row, so a warp instruction touches 4 (bf16) or 2 (fp32) cache lines).
// Steps past seqlen and channels past dim read as zero.
template <typename IT>
__device__ __forceinline__ void conv_load_cols(IT* dst, const IT* slab, int64_t dim_stride, int t0, int ncols, int c0,
                                               int dim, int L, bool vec) {
  constexpr int VW = 16 / sizeof(IT);
  constexpr int CH = kConvT / VW;
  constexpr int P = conv_pitch<IT>();
  for (int i = threadIdx.x; i < kConvC * CH; i += kConvThreads) {
    const int r = i / CH, ch = (i % CH) * VW;
    const int c = c0 + r, t = t0 + ch;
    uint4 pk = make_uint4(0u, 0u, 0u, 0u);
    IT* e = reinterpret_cast<IT*>(&pk);
    if (c < dim) {
      const IT* src = slab + (int64_t)c * dim_stride + t;
      if (vec && t + VW <= L) {
        pk = *reinterpret_cast<const uint4*>(src);
      } else {
#pragma unroll
        for (int j = 0; j < VW; ++j)
          if (t + j < L) e[j] = src[j];
      }
    }
    *reinterpret_cast<uint4*>(dst + r * P + ch) = pk;
  }
  const int halo = ncols - kConvT;  // 0 .. K-1 extra steps after the tile
  for (int i = threadIdx.x; i < kConvC * halo; i += kConvThreads) {
    const int r = i / halo, j = i % halo;
    const int c = c0 + r, t = t0 + kConvT + j;
    dst[r * P + kConvT + j] = (c < dim && t < L) ? slab[(int64_t)c * dim_stride + t] : from_f<IT>(0.f);
  }
}

// Store a [64 channels][64 steps] staging tile to (c0, t0) of a (dim, seqlen) slab with
// row-contiguous 16-byte stores; steps past seqlen and channels past dim are skipped.
template <typename IT>
__device__ __forceinline__ void conv_store_cols(IT* slab, int64_t dim_stride, const IT* src, int t0, int c0, int dim,
                                                int L, bool vec) {
  constexpr int VW = 16 / sizeof(IT);
  constexpr int CH = kConvT / VW;
  constexpr int P = conv_pitch<IT>();
  for (int i = threadIdx.x; i < kConvC * CH; i += kConvThreads) {
    const int r = i / CH, ch = (i % CH) * VW;
    const int c = c0 + r, t = t0 + ch;
    if (c >= dim || t >= L) continue;
    IT* dst = slab + (int64_t)c * dim_stride + t;
    const uint4 pk = *reinterpret_cast<const uint4*>(src + r * P + ch);
    if (vec && t + VW <= L) {
      *reinterpret_cast<uint4*>(dst) = pk;
    } else {
      const IT* e = reinterpret_cast<const IT*>(&pk);
#pragma unroll
      for (int j = 0; j < VW; ++j)
        if (t + j < L) dst[j] = e[j];
    }
  }
}

// 16 consecutive steps of one channel of a staging tile, as float / from float (16-byte
// shared accesses; lanes hold consecutive channels).
template <typename IT>
__device__ __forceinline__ void tile_get16(const IT* row, float* v) {
  constexpr int VW = 16 / sizeof(IT);
#pragma unroll
  for (int q = 0; q < kConvTPT / VW; ++q) {
    const uint4 pk = *reinterpret_cast<const uint4*>(row + q * VW);
    const IT* e = reinterpret_cast<const IT*>(&pk);
#pragma unroll
    for (int j = 0; j < VW; ++j) v[q * VW + j] = to_f<IT>(e[j]);
  }
}
template <typename IT>
__device__ __forceinline__ void tile_put16(IT* row, const float* v) {
  constexpr int VW = 16 / sizeof(IT);
#pragma unroll
  for (int q = 0; q < kConvTPT / VW; ++q) {
    uint4 pk;
    IT* e = reinterpret_cast<IT*>(&pk);
#pragma unroll
    for (int j = 0; j < VW; ++j) e[j] = from_f<IT>(v[q * VW + j]);
    *reinterpret_cast<uint4*>(row + q * VW) = pk;
  }
}

__device__ __forceinline__ float silu_f(float p) { return p * sigmoid_fast(p); }

template <typename IT, int K>
struct ConvFwdSmem {
  alignas(16) IT x[kConvT + K - 1][kConvC];       // [step][channel], as read from (seqlen, dim)
  alignas(16) IT z[kConvT][kConvC];
  alignas(16) IT u[kConvC][conv_pitch<IT>()];     // [channel][step], as written to (dim, seqlen)
  alignas(16) IT zt[kConvC][conv_pitch<IT>()];
};

template <typename IT, int K, bool kHasZ>
__global__ void __launch_bounds__(kConvThreads) conv_fwd_kernel(const __grid_constant__ ConvK P) {
  extern __shared__ __align__(16) unsigned char conv_smem[];
  ConvFwdSmem<IT, K>& sm = *reinterpret_cast<ConvFwdSmem<IT, K>*>(conv_smem);
  const ss_conv_args& a = P.a;
  const int c0 = (blockIdx.x % P.nc) * kConvC, t0 = ((blockIdx.x / P.nc) % P.nt) * kConvT;
  const int b = blockIdx.x / P.nc / P.nt;
  const int L = a.seqlen, dim = a.dim;
  const IT* xb = (const IT*)a.x + (int64_t)b * a.x_batch_stride;
  const float* state_b = a.state_in != nullptr ? a.state_in + (int64_t)b * dim * (K - 1) : nullptr;
  conv_load_rows<IT, K>(&sm.x[0][0], kConvT + K - 1, xb, a.x_seq_stride, t0 - (K - 1), c0, dim, L, state_b,
                        P.vec_x);
  if constexpr (kHasZ)
    conv_load_rows<IT, 1>(&sm.z[0][0], kConvT, (const IT*)a.z + (int64_t)b * a.z_batch_stride, a.z_seq_stride, t0,
                          c0, dim, L, nullptr, P.vec_z);
  __syncthreads();

  const int cl = threadIdx.x % kConvC, g = threadIdx.x / kConvC;
  const int c = c0 + cl, tb = g * kConvTPT;
  {
    float w[K];
#pragma unroll
    for (int k = 0; k < K; ++k) w[k] = c < dim ? a.weight[(int64_t)c * K + k] : 0.f;
    const float bias = (c < dim && a.bias != nullptr) ? a.bias[c] : 0.f;
    float v[kConvTPT];
#pragma unroll
    for (int i = 0; i < kConvTPT; ++i) {
      float p = bias;
#pragma unroll
      for (int k = 0; k < K; ++k) p = fmaf(w[k], to_f<IT>(sm.x[tb + i + k][cl]), p);
      v[i] = a.silu ? silu_f(p) : p;
    }
    tile_put16<IT>(&sm.u[cl][tb], v);
    if constexpr (kHasZ) {
#pragma unroll
      for (int i = 0; i < kConvTPT; ++i) v[i] = to_f<IT>(sm.z[tb + i][cl]);
      tile_put16<IT>(&sm.zt[cl][tb], v);
    }
  }
  __syncthreads();
  conv_store_cols<IT>((IT*)a.u + (int64_t)b * a.u_batch_stride, a.u_dim_stride, &sm.u[0][0], t0, c0, dim, L,
                      P.vec_u);
  if constexpr (kHasZ)
    conv_store_cols<IT>((IT*)a.zt + (int64_t)b * a.zt_batch_stride, a.zt_dim_stride, &sm.zt[0][0], t0, c0, dim, L,
                        P.vec_zt);
  // the last K-1 inputs of the sequence become the state for a following chunk or decode
  if (K > 1 && a.state_out != nullptr && t0 + kConvT >= L && g == 0 && c < dim) {
#pragma unroll
    for (int j = 0; j < K - 1; ++j) {
      const int t = L - (K - 1) + j;  // an input of this call, or of the state when seqlen < K-1
      const float v = t >= 0 ? to_f<IT>(xb[(int64_t)t * a.x_seq_stride + c])
                             : (state_b != nullptr ? state_b[(int64_t)c * (K - 1) + (t + K - 1)] : 0.f);
      a.state_out[((int64_t)b * dim + c) * (K - 1) + j] = v;
    }
  }
}

// ~41 KB (bf16, K = 4): five CTAs per SM.  dpre is kept at the I/O precision (it only feeds
// dx, which is stored at that precision; dweight / dbias accumulate in fp32 registers), and
// the dx / dz staging tile reuses the du tile, which is dead once dpre is formed.
template <typename IT, int K>
struct ConvBwdSmem {
  alignas(16) IT x[kConvT + 2 * (K - 1)][kConvC];  // steps t0-(K-1) .. t0+63+(K-1)
  union {
    alignas(16) IT du[kConvC][conv_pitch<IT>()];   // [channel][step t0 .. t0+63+(K-1)]
    alignas(16) IT out[kConvT][kConvC];            // dx (then dz) staged for row stores
  };
  alignas(16) IT dzt[kConvC][conv_pitch<IT>()];
  alignas(16) IT dp[kConvT + K - 1][kConvC];       // dpre for steps t0 .. t0+63+(K-1)
  float red[kConvThreads / kConvC][kConvC][K + 1];
};

template <typename IT, int K, bool kHasZ>
__global__ void __launch_bounds__(kConvThreads) conv_bwd_kernel(const __grid_constant__ ConvBwdK P) {
  extern __shared__ __align__(16) unsigned char conv_smem[];
  ConvBwdSmem<IT, K>& sm = *reinterpret_cast<ConvBwdSmem<IT, K>*>(conv_smem);
  const ss_conv_bwd_args& a = P.a;
  const ss_conv_args& f = a.f;
  const int c0 = (blockIdx.x % P.nc) * kConvC, t0 = ((blockIdx.x / P.nc) % P.nt) * kConvT;
  const int b = blockIdx.x / P.nc / P.nt;
  const int L = f.seqlen, dim = f.dim;
  const IT* xb = (const IT*)f.x + (int64_t)b * f.x_batch_stride;
  const float* state_b = f.state_in != nullptr ? f.state_in + (int64_t)b * dim * (K - 1) : nullptr;
  conv_load_rows<IT, K>(&sm.x[0][0], kConvT + 2 * (K - 1), xb, f.x_seq_stride, t0 - (K - 1), c0, dim, L, state_b,
                        P.vec_x);
  conv_load_cols<IT>(&sm.du[0][0], (const IT*)a.du + (int64_t)b * a.du_batch_stride, a.du_dim_stride, t0,
                     kConvT + K - 1, c0, dim, L, P.vec_du);
  if constexpr (kHasZ)
    conv_load_cols<IT>(&sm.dzt[0][0], (const IT*)a.dzt + (int64_t)b * a.dzt_batch_stride, a.dzt_dim_stride, t0,
                       kConvT, c0, dim, L, P.vec_dzt);
  __syncthreads();

  const int cl = threadIdx.x % kConvC, g = threadIdx.x / kConvC;
  const int c = c0 + cl, tb = g * kConvTPT;
  const bool cok = c < dim;
  float w[K];
#pragma unroll
  for (int k = 0; k < K; ++k) w[k] = cok ? f.weight[(int64_t)c * K + k] : 0.f;
  const float bias = (cok && f.bias != nullptr) ? f.bias[c] : 0.f;

  // dpre for this thread's 16 steps (and, for the last thread row, the K-1 steps after the tile)
  float dw[K], db = 0.f;
#pragma unroll
  for (int k = 0; k < K; ++k) dw[k] = 0.f;
  {
    float duv[kConvTPT];
    tile_get16<IT>(&sm.du[cl][tb], duv);  // zero past seqlen and past dim
#pragma unroll
    for (int i = 0; i < kConvTPT; ++i) {
      float p = bias;
#pragma unroll
      for (int k = 0; k < K; ++k) p = fmaf(w[k], to_f<IT>(sm.x[tb + i + k][cl]), p);
      float d = 0.f;
      if (f.silu) {
        const float s = sigmoid_fast(p);
        d = duv[i] * s * fmaf(p, 1.f - s, 1.f);
      } else {
        d = duv[i];
      }
      sm.dp[tb + i][cl] = from_f<IT>(d);
      db += d;
#pragma unroll
      for (int k = 0; k < K; ++k) dw[k] = fmaf(d, to_f<IT>(sm.x[tb + i + k][cl]), dw[k]);
    }
    if (g == kConvThreads / kConvC - 1) {
#pragma unroll
      for (int j = 0; j < K - 1; ++j) {
        const int r = kConvT + j, t = t0 + r;
        float d = 0.f;
        if (cok && t < L) {
          float p = bias;
#pragma unroll
          for (int k = 0; k < K; ++k) p = fmaf(w[k], to_f<IT>(sm.x[r + k][cl]), p);
          const float dv = to_f<IT>(sm.du[cl][r]);
          if (f.silu) {
            const float s = sigmoid_fast(p);
            d = dv * s * fmaf(p, 1.f - s, 1.f);
          } else {
            d = dv;
          }
        }
        sm.dp[r][cl] = from_f<IT>(d);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < K; ++k) sm.red[g][cl][k] = dw[k];
  sm.red[g][cl][K] = db;
  __syncthreads();

  // dx[t] = sum_k w[k] dpre[t + (K-1) - k], staged as a [t][c] tile for row stores
#pragma unroll
  for (int i = 0; i < kConvTPT; ++i) {
    float s = 0.f;
#pragma unroll
    for (int k = 0; k < K; ++k) s = fmaf(w[k], to_f<IT>(sm.dp[tb + i + (K - 1) - k][cl]), s);
    sm.out[tb + i][cl] = from_f<IT>(s);
  }
  if (threadIdx.x < kConvC && c0 + (int)threadIdx.x < dim) {
    const int cc = c0 + threadIdx.x;
#pragma unroll
    for (int k = 0; k <= K; ++k) {
      float s = 0.f;
#pragma unroll
      for (int r = 0; r < kConvThreads / kConvC; ++r) s += sm.red[r][threadIdx.x][k];
      if (k < K) atomicAdd(a.dweight + (int64_t)cc * K + k, s);
      else if (a.dbias != nullptr) atomicAdd(a.dbias + cc, s);
    }
  }
  __syncthreads();
  conv_store_rows<IT>((IT*)a.dx + (int64_t)b * a.dx_batch_stride, a.dx_seq_stride, &sm.out[0][0], t0, c0, dim, L,
                      P.vec_dx);
  if constexpr (kHasZ) {
    __syncthreads();
    float v[kConvTPT];
    tile_get16<IT>(&sm.dzt[cl][tb], v);
#pragma unroll
    for (int i = 0; i < kConvTPT; ++i) sm.out[tb + i][cl] = from_f<IT>(v[i]);
    __syncthreads();
    conv_store_rows<IT>((IT*)a.dz + (int64_t)b * a.dz_batch_stride, a.dz_seq_stride, &sm.out[0][0], t0, c0, dim, L,
                        P.vec_dz);
  }
}

// One decode step: window = [state (oldest first), x]; u = silu(bias + w . window);
// state <- window[1:].  One thread per (batch, channel).
template <typename IT, int K>
__global__ void __launch_bounds__(128) conv_step_kernel(const __grid_constant__ ss_conv_step_args a, int ncb) {
  const int c = (blockIdx.x % ncb) * 128 + threadIdx.x, b = blockIdx.x / ncb;
  if (c >= a.dim) return;
  float win[K];
  float* st = a.state + (int64_t)b * a.state_batch_stride + (int64_t)c * (K - 1);
#pragma unroll
  for (int k = 0; k < K - 1; ++k) win[k] = st[k];
  win[K - 1] = to_f<IT>(((const IT*)a.x)[(int64_t)b * a.x_batch_stride + c]);
  float p = a.bias != nullptr ? a.bias[c] : 0.f;
#pragma unroll
  for (int k = 0; k < K; ++k) p = fmaf(a.weight[(int64_t)c * K + k], win[k], p);
  ((IT*)a.u)[(int64_t)b * a.u_batch_stride + c] = from_f<IT>(a.silu ? silu_f(p) : p);
#pragma unroll
  for (int k = 0; k < K - 1; ++k) st[k] = win[k + 1];
}

}  // namespace ssb
