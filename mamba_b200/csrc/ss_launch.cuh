// Kernel launchers: compile-time dispatch over the warp count (dstate <= 4, 8, 16),
// variable / constant B and C, the z gate and the load path (TMA ring or synchronous).
// Instantiated once per I/O dtype.
#pragma once
#include "ss_fwd.cuh"
#include "ss_bwd.cuh"
#include "ss_step.cuh"

namespace ssb {

inline int warps_for(int dstate) { return dstate <= 4 ? 1 : (dstate <= 8 ? 2 : 4); }

template <typename K, typename Arg>
static cudaError_t launch_dyn(K kernel, dim3 grid, int threads, size_t smem, cudaStream_t st, const Arg& P) {
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  kernel<<<grid, threads, smem, st>>>(P);
  return cudaGetLastError();
}

template <typename IT, int NW, bool VB, bool VC, bool Z>
static cudaError_t fwd_go(const FwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  const size_t smem = sizeof(FwdSmem<IT, NW, VB, VC, Z>);
  if (tma) return launch_dyn(ss_fwd_kernel<IT, NW, VB, VC, Z, true>, grid, 32 * NW, smem, st, P);
  return launch_dyn(ss_fwd_kernel<IT, NW, VB, VC, Z, false>, grid, 32 * NW, smem, st, P);
}
template <typename IT, int NW, bool VB, bool VC>
static cudaError_t fwd_z(const FwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  return P.a.z != nullptr ? fwd_go<IT, NW, VB, VC, true>(P, grid, st, tma)
                          : fwd_go<IT, NW, VB, VC, false>(P, grid, st, tma);
}
template <typename IT, int NW>
static cudaError_t fwd_bc(const FwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  const bool vb = P.a.var_B != 0, vc = P.a.var_C != 0;
  if (vb && vc) return fwd_z<IT, NW, true, true>(P, grid, st, tma);
  if (vb) return fwd_z<IT, NW, true, false>(P, grid, st, tma);
  if (vc) return fwd_z<IT, NW, false, true>(P, grid, st, tma);
  return fwd_z<IT, NW, false, false>(P, grid, st, tma);
}
template <typename IT>
cudaError_t launch_fwd(const FwdK& P, cudaStream_t st, bool tma) {
  dim3 grid(P.a.ngroups * P.tpg, P.a.batch);
  switch (warps_for(P.a.dstate)) {
    case 1: return fwd_bc<IT, 1>(P, grid, st, tma);
    case 2: return fwd_bc<IT, 2>(P, grid, st, tma);
    default: return fwd_bc<IT, 4>(P, grid, st, tma);
  }
}

template <typename IT, int NW, bool VB, bool VC, bool Z>
static cudaError_t bwd_go(const BwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  const size_t smem = sizeof(BwdSmem<IT, NW, VB, VC, Z>);
  if (tma) return launch_dyn(ss_bwd_kernel<IT, NW, VB, VC, Z, true>, grid, 32 * NW, smem, st, P);
  return launch_dyn(ss_bwd_kernel<IT, NW, VB, VC, Z, false>, grid, 32 * NW, smem, st, P);
}
template <typename IT, int NW, bool VB, bool VC>
static cudaError_t bwd_z(const BwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  return P.a.f.z != nullptr ? bwd_go<IT, NW, VB, VC, true>(P, grid, st, tma)
                            : bwd_go<IT, NW, VB, VC, false>(P, grid, st, tma);
}
template <typename IT, int NW>
static cudaError_t bwd_bc(const BwdK& P, dim3 grid, cudaStream_t st, bool tma) {
  const bool vb = P.a.f.var_B != 0, vc = P.a.f.var_C != 0;
  if (vb && vc) return bwd_z<IT, NW, true, true>(P, grid, st, tma);
  if (vb) return bwd_z<IT, NW, true, false>(P, grid, st, tma);
  if (vc) return bwd_z<IT, NW, false, true>(P, grid, st, tma);
  return bwd_z<IT, NW, false, false>(P, grid, st, tma);
}
template <typename IT>
cudaError_t launch_bwd(const BwdK& P, cudaStream_t st, bool tma) {
  dim3 grid(P.a.f.ngroups * P.tpg, P.a.f.batch);
  switch (warps_for(P.a.f.dstate)) {
    case 1: return bwd_bc<IT, 1>(P, grid, st, tma);
    case 2: return bwd_bc<IT, 2>(P, grid, st, tma);
    default: return bwd_bc<IT, 4>(P, grid, st, tma);
  }
}

template <typename IT>
cudaError_t launch_step(const ss_step_args& a, cudaStream_t st) {
  const int tpc = warps_for(a.dstate);  // threads per channel = ceil(dstate / 4), as 1/2/4
  const int cpb = 128 / tpc;
  dim3 grid((a.dim + cpb - 1) / cpb, a.batch);
  if (tpc == 1) ss_step_kernel<IT, 1><<<grid, 128, 0, st>>>(a);
  else if (tpc == 2) ss_step_kernel<IT, 2><<<grid, 128, 0, st>>>(a);
  else ss_step_kernel<IT, 4><<<grid, 128, 0, st>>>(a);
  return cudaGetLastError();
}

}  // namespace ssb

#define SSB_INSTANTIATE(IT)                                                          \
  namespace ssb {                                                                    \
  template cudaError_t launch_fwd<IT>(const FwdK&, cudaStream_t, bool);              \
  template cudaError_t launch_bwd<IT>(const BwdK&, cudaStream_t, bool);              \
  template cudaError_t launch_step<IT>(const ss_step_args&, cudaStream_t);           \
  }
