// Kernel launchers: compile-time dispatch over the warp count (dstate <= 4, 8, 16, or state
// groups of 16 above that), variable / constant B and C, the z gate and the load path (TMA
// ring or synchronous).  Instantiated once per I/O dtype.
#pragma once
#include "ss_fwd.cuh"
#include "ss_bwd.cuh"
#include "ss_chunk.cuh"
#include "ss_step.cuh"

namespace ssb {

inline int warps_for(int dstate) { return dstate <= 4 ? 1 : (dstate <= 8 ? 2 : 4); }

// pdl: launch with programmatic stream serialization, so the kernel may start while the one
// ahead of it in the stream still runs (the kernel itself waits, griddep_wait, where it reads that
// kernel's results).
template <typename K, typename Arg>
static cudaError_t launch_dyn(K kernel, dim3 grid, int threads, size_t smem, cudaStream_t st, const Arg& P,
                              bool pdl = false) {
  cudaError_t e = ensure_smem_limit(reinterpret_cast<const void*>(kernel), smem);
  if (e != cudaSuccess) return e;
  if (!pdl) {
    kernel<<<grid, threads, smem, st>>>(P);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, P);
}

// ---- forward
template <typename IT, int NW, bool VB, bool VC, bool Z, bool M>
static cudaError_t fwd_go(const FwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  const size_t smem = sizeof(FwdSmem<IT, NW, VB, VC, Z>);
  const bool pdl = P.nchunk > 1;  // follows ss_fwd_chunk_kernel in the stream
  if constexpr (!M) {  // (b, L, d) tensors: TMA only, dstate <= 16 (checked on the host)
    if (P.a.layout == SS_LAYOUT_BLD)
      return launch_dyn(ss_fwd_kernel<IT, NW, VB, VC, Z, true, false, true>, grid, 32 * NW, smem, st, P, pdl);
  }
  if (tma) return launch_dyn(ss_fwd_kernel<IT, NW, VB, VC, Z, true, M>, grid, 32 * NW, smem, st, P, pdl);
  return launch_dyn(ss_fwd_kernel<IT, NW, VB, VC, Z, false, M>, grid, 32 * NW, smem, st, P, pdl);
}
template <typename IT, int NW, bool VB, bool VC, bool M>
static cudaError_t fwd_z(const FwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  if constexpr (M) return fwd_go<IT, NW, VB, VC, false, true>(P, grid, st, tma);  // gate in the finish
  else
    return P.a.z != nullptr ? fwd_go<IT, NW, VB, VC, true, false>(P, grid, st, tma)
                            : fwd_go<IT, NW, VB, VC, false, false>(P, grid, st, tma);
}
template <typename IT, int NW, bool M>
static cudaError_t fwd_bc(const FwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  const bool vb = P.a.var_B != 0, vc = P.a.var_C != 0;
  if (vb && vc) return fwd_z<IT, NW, true, true, M>(P, grid, st, tma);
  if (vb) return fwd_z<IT, NW, true, false, M>(P, grid, st, tma);
  if (vc) return fwd_z<IT, NW, false, true, M>(P, grid, st, tma);
  return fwd_z<IT, NW, false, false, M>(P, grid, st, tma);
}
// chunk summaries of the forward (time chunks 0 .. nchunk - 2)
template <typename IT, int NW, bool VB>
static cudaError_t fwd_chunk_go(const FwdK& P, cudaStream_t st) {
  dim3 grid((unsigned)((int64_t)P.a.batch * P.nct * (P.nchunk - 1)));
  const size_t smem = sizeof(FwdChunkSmem<IT, NW, VB>);
  if (P.a.layout == SS_LAYOUT_BLD) return launch_dyn(ss_fwd_chunk_kernel<IT, NW, VB, true>, grid, 32 * NW, smem, st, P);
  return launch_dyn(ss_fwd_chunk_kernel<IT, NW, VB, false>, grid, 32 * NW, smem, st, P);
}
template <typename IT, int NW>
static cudaError_t fwd_chunk_b(const FwdK& P, cudaStream_t st) {
  return P.a.var_B ? fwd_chunk_go<IT, NW, true>(P, st) : fwd_chunk_go<IT, NW, false>(P, st);
}
template <typename IT>
static cudaError_t fwd_chunks(const FwdK& P, cudaStream_t st) {
  switch (warps_for(P.a.dstate)) {
    case 1: return fwd_chunk_b<IT, 1>(P, st);
    case 2: return fwd_chunk_b<IT, 2>(P, st);
    default: return fwd_chunk_b<IT, 4>(P, st);
  }
}

template <typename IT>
cudaError_t launch_fwd(const FwdK& P, cudaStream_t st, bool tma) {
  const ss_fwd_args& a = P.a;
  // sizes checked on the host; nchunk > 1 only with TMA and dstate <= 16
  dim3 grid((unsigned)((int64_t)a.batch * P.nsg * P.nct * P.nchunk));
  if (P.nsg > 1) {
    // state groups: partial sums meet in the workspace, then the gate is applied
    cudaError_t e = cudaMemsetAsync(a.work, 0, (size_t)a.batch * a.dim * (size_t)a.seqlen * sizeof(float), st);
    if (e != cudaSuccess) return e;
    e = fwd_bc<IT, 4, true>(P, grid, st, tma);
    if (e != cudaSuccess) return e;
    const int nlc = (a.seqlen + 255) / 256;
    fwd_finish_kernel<IT><<<(unsigned)((int64_t)a.batch * a.dim * nlc), 256, 0, st>>>(a, nlc);
    return cudaGetLastError();
  }
  if (P.nchunk > 1) {
    cudaError_t e = fwd_chunks<IT>(P, st);
    if (e != cudaSuccess) return e;
  }
  switch (warps_for(a.dstate)) {
    case 1: return fwd_bc<IT, 1, false>(P, grid, st, tma);
    case 2: return fwd_bc<IT, 2, false>(P, grid, st, tma);
    default: return fwd_bc<IT, 4, false>(P, grid, st, tma);
  }
}

// ---- backward
template <typename IT, int NW, bool VB, bool VC, bool Z, bool M>
static cudaError_t bwd_go(const BwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  const size_t smem = sizeof(BwdSmem<IT, NW, VB, VC, Z>);
  // follows ss_bwd_carry_kernel, or the zeroing kernel (zero_dep), in the stream
  const bool pdl = P.nchunk > 1 || P.zero_dep != 0;
  if constexpr (!M) {  // (b, L, d) tensors: TMA only, dstate <= 16 (checked on the host)
    if (P.a.f.layout == SS_LAYOUT_BLD)
      return launch_dyn(ss_bwd_kernel<IT, NW, VB, VC, Z, true, false, true>, grid, 32 * NW, smem, st, P, pdl);
  }
  if (tma) return launch_dyn(ss_bwd_kernel<IT, NW, VB, VC, Z, true, M>, grid, 32 * NW, smem, st, P, pdl);
  return launch_dyn(ss_bwd_kernel<IT, NW, VB, VC, Z, false, M>, grid, 32 * NW, smem, st, P, pdl);
}
template <typename IT, int NW, bool VB, bool VC, bool M>
static cudaError_t bwd_z(const BwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  return P.a.f.z != nullptr ? bwd_go<IT, NW, VB, VC, true, M>(P, grid, st, tma)
                            : bwd_go<IT, NW, VB, VC, false, M>(P, grid, st, tma);
}
template <typename IT, int NW, bool M>
static cudaError_t bwd_bc(const BwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  const bool vb = P.a.f.var_B != 0, vc = P.a.f.var_C != 0;
  if (vb && vc) return bwd_z<IT, NW, true, true, M>(P, grid, st, tma);
  if (vb) return bwd_z<IT, NW, true, false, M>(P, grid, st, tma);
  if (vc) return bwd_z<IT, NW, false, true, M>(P, grid, st, tma);
  return bwd_z<IT, NW, false, false, M>(P, grid, st, tma);
}
// chunk carries of the backward (time chunks 1 .. nchunk - 1)
template <typename IT, int NW, bool VC, bool Z>
static cudaError_t bwd_carry_go(const BwdK& P, cudaStream_t st) {
  dim3 grid((unsigned)((int64_t)P.a.f.batch * P.nct * (P.nchunk - 1)));
  const size_t smem = sizeof(BwdCarrySmem<IT, NW, VC, Z>);
  if (P.a.f.layout == SS_LAYOUT_BLD)
    return launch_dyn(ss_bwd_carry_kernel<IT, NW, VC, Z, true>, grid, 32 * NW, smem, st, P);
  return launch_dyn(ss_bwd_carry_kernel<IT, NW, VC, Z, false>, grid, 32 * NW, smem, st, P);
}
template <typename IT, int NW>
static cudaError_t bwd_carry_cz(const BwdK& P, cudaStream_t st) {
  const bool vc = P.a.f.var_C != 0, z = P.a.f.z != nullptr;
  if (vc) return z ? bwd_carry_go<IT, NW, true, true>(P, st) : bwd_carry_go<IT, NW, true, false>(P, st);
  return z ? bwd_carry_go<IT, NW, false, true>(P, st) : bwd_carry_go<IT, NW, false, false>(P, st);
}
template <typename IT>
static cudaError_t bwd_carries(const BwdK& P, cudaStream_t st) {
  switch (warps_for(P.a.f.dstate)) {
    case 1: return bwd_carry_cz<IT, 1>(P, st);
    case 2: return bwd_carry_cz<IT, 2>(P, st);
    default: return bwd_carry_cz<IT, 4>(P, st);
  }
}

template <typename IT>
cudaError_t launch_bwd(const BwdK& P, cudaStream_t st, bool tma) {
  const ss_fwd_args& f = P.a.f;
  // sizes checked on the host; nchunk > 1 only with TMA and dstate <= 16
  dim3 grid((unsigned)((int64_t)f.batch * P.nsg * P.nct * P.nchunk));
  if (P.nsg > 1) {
    cudaError_t e =
        cudaMemsetAsync(f.work, 0, 2 * (size_t)f.batch * f.dim * (size_t)f.seqlen * sizeof(float), st);
    if (e != cudaSuccess) return e;
    e = bwd_bc<IT, 4, true>(P, grid, st, tma);
    if (e != cudaSuccess) return e;
    const int nlc = (f.seqlen + 255) / 256;
    bwd_finish_kernel<IT><<<(unsigned)((int64_t)f.batch * f.dim * nlc), 256, 0, st>>>(P.a, nlc);
    return cudaGetLastError();
  }
  if (P.nchunk > 1) {
    cudaError_t e = bwd_carries<IT>(P, st);
    if (e != cudaSuccess) return e;
  }
  switch (warps_for(f.dstate)) {
    case 1: return bwd_bc<IT, 1, false>(P, grid, st, tma);
    case 2: return bwd_bc<IT, 2, false>(P, grid, st, tma);
    default: return bwd_bc<IT, 4, false>(P, grid, st, tma);
  }
}

// ---- decode step
template <typename IT, int TPC, int R>
static cudaError_t step_go(const ss_step_args& a, cudaStream_t st) {
  constexpr int CPB = 128 / TPC;
  const int nblk = (a.dim + CPB - 1) / CPB;
  ss_step_kernel<IT, TPC, R><<<(unsigned)((int64_t)a.batch * nblk), 128, 0, st>>>(a, nblk);
  return cudaGetLastError();
}
template <typename IT>
cudaError_t launch_step(const ss_step_args& a, cudaStream_t st) {
  int tpc, chunks;
  step_shape(a.dstate, tpc, chunks);
  switch (tpc) {
    case 1: return step_go<IT, 1, 1>(a, st);
    case 2: return step_go<IT, 2, 1>(a, st);
    case 4: return step_go<IT, 4, 1>(a, st);
    case 8: return step_go<IT, 8, 1>(a, st);
    case 16: return step_go<IT, 16, 1>(a, st);
    default: return chunks == 1 ? step_go<IT, 32, 1>(a, st) : step_go<IT, 32, 2>(a, st);
  }
}

}  // namespace ssb

#define SSB_INSTANTIATE(IT)                                                          \
  namespace ssb {                                                                    \
  template cudaError_t launch_fwd<IT>(const FwdK&, cudaStream_t, bool);              \
  template cudaError_t launch_bwd<IT>(const BwdK&, cudaStream_t, bool);              \
  template cudaError_t launch_step<IT>(const ss_step_args&, cudaStream_t);           \
  }
