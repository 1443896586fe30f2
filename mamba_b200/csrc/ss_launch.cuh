// Kernel launchers: compile-time dispatch over the warp count (dstate <= 4, 8, 16),
// variable / constant B and C, and the z gate.  Instantiated once per I/O dtype.
#pragma once
#include "ss_fwd.cuh"
#include "ss_bwd.cuh"
#include "ss_step.cuh"

namespace ssb {

inline int warps_for(int dstate) { return dstate <= 4 ? 1 : (dstate <= 8 ? 2 : 4); }

template <typename IT, int NW, bool VB, bool VC>
static void fwd_z(const FwdK& P, dim3 grid, cudaStream_t st) {
  if (P.a.z != nullptr) ss_fwd_kernel<IT, NW, VB, VC, true><<<grid, 32 * NW, 0, st>>>(P);
  else ss_fwd_kernel<IT, NW, VB, VC, false><<<grid, 32 * NW, 0, st>>>(P);
}
template <typename IT, int NW>
static void fwd_bc(const FwdK& P, dim3 grid, cudaStream_t st) {
  const bool vb = P.a.var_B != 0, vc = P.a.var_C != 0;
  if (vb && vc) fwd_z<IT, NW, true, true>(P, grid, st);
  else if (vb) fwd_z<IT, NW, true, false>(P, grid, st);
  else if (vc) fwd_z<IT, NW, false, true>(P, grid, st);
  else fwd_z<IT, NW, false, false>(P, grid, st);
}
template <typename IT>
cudaError_t launch_fwd(const FwdK& P, cudaStream_t st) {
  dim3 grid(P.a.ngroups * P.tpg, P.a.batch);
  switch (warps_for(P.a.dstate)) {
    case 1: fwd_bc<IT, 1>(P, grid, st); break;
    case 2: fwd_bc<IT, 2>(P, grid, st); break;
    default: fwd_bc<IT, 4>(P, grid, st); break;
  }
  return cudaGetLastError();
}

template <typename IT, int NW, bool VB, bool VC>
static void bwd_z(const BwdK& P, dim3 grid, cudaStream_t st) {
  if (P.a.f.z != nullptr) ss_bwd_kernel<IT, NW, VB, VC, true><<<grid, 32 * NW, 0, st>>>(P);
  else ss_bwd_kernel<IT, NW, VB, VC, false><<<grid, 32 * NW, 0, st>>>(P);
}
template <typename IT, int NW>
static void bwd_bc(const BwdK& P, dim3 grid, cudaStream_t st) {
  const bool vb = P.a.f.var_B != 0, vc = P.a.f.var_C != 0;
  if (vb && vc) bwd_z<IT, NW, true, true>(P, grid, st);
  else if (vb) bwd_z<IT, NW, true, false>(P, grid, st);
  else if (vc) bwd_z<IT, NW, false, true>(P, grid, st);
  else bwd_z<IT, NW, false, false>(P, grid, st);
}
template <typename IT>
cudaError_t launch_bwd(const BwdK& P, cudaStream_t st) {
  dim3 grid(P.a.f.ngroups * P.tpg, P.a.f.batch);
  switch (warps_for(P.a.f.dstate)) {
    case 1: bwd_bc<IT, 1>(P, grid, st); break;
    case 2: bwd_bc<IT, 2>(P, grid, st); break;
    default: bwd_bc<IT, 4>(P, grid, st); break;
  }
  return cudaGetLastError();
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
  template cudaError_t launch_fwd<IT>(const FwdK&, cudaStream_t);                    \
  template cudaError_t launch_bwd<IT>(const BwdK&, cudaStream_t);                    \
  template cudaError_t launch_step<IT>(const ss_step_args&, cudaStream_t);           \
  }
