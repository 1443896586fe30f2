// C ABI of libmamba_b200_ss.so: argument validation, derived launch parameters and
// dtype dispatch.  The reference has no input checks at all (its binding,
// csrc/selective_scan/selective_scan.cpp:184-329, passes raw pointers straight through);
// here every call is checked first and reports a status code instead of faulting.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/mamba_b200_ss.h"
#include "ss_common.cuh"

namespace ssb {
template <typename IT> cudaError_t launch_fwd(const FwdK&, cudaStream_t);
template <typename IT> cudaError_t launch_bwd(const BwdK&, cudaStream_t);
template <typename IT> cudaError_t launch_step(const ss_step_args&, cudaStream_t);
}  // namespace ssb

namespace {

thread_local int g_last_cuda = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return SS_OK;
  g_last_cuda = (int)e;
  return SS_ERR_CUDA;
}

size_t esize(int dt) { return dt == SS_F32 ? 4 : 2; }
bool dtype_ok(int dt) { return dt == SS_F32 || dt == SS_BF16 || dt == SS_F16; }

// every (batch, channel) row of a (batch, dim, seqlen) view starts 16-byte aligned
bool rows16(const void* p, int64_t bs, int64_t ds, size_t es) {
  return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && ((bs * (int64_t)es) & 15) == 0 &&
         ((ds * (int64_t)es) & 15) == 0;
}

int check_fwd(const ss_fwd_args* a) {
  if (a == nullptr) return SS_ERR_INVALID;
  if (a->batch < 0 || a->dim < 1 || a->seqlen < 0 || a->dstate < 1 || a->ngroups < 1) return SS_ERR_INVALID;
  if (a->dim % a->ngroups != 0) return SS_ERR_INVALID;
  if (a->batch > 65535) return SS_ERR_UNSUPPORTED;
  if (a->dstate > SS_MAX_DSTATE) return SS_ERR_UNSUPPORTED;
  if (!dtype_ok(a->io_dtype) || !dtype_ok(a->bc_dtype)) return SS_ERR_UNSUPPORTED;
  if (a->bc_dtype != SS_F32 && a->bc_dtype != a->io_dtype) return SS_ERR_UNSUPPORTED;
  if (!a->u || !a->delta || !a->A || !a->B || !a->C) return SS_ERR_INVALID;
  if (a->u_batch_stride < 0 || a->u_dim_stride < 0 || a->delta_batch_stride < 0 || a->delta_dim_stride < 0)
    return SS_ERR_INVALID;
  if (a->z && (a->z_batch_stride < 0 || a->z_dim_stride < 0)) return SS_ERR_INVALID;
  return SS_OK;
}

void derive(const ss_fwd_args& a, int& dpg, int& tpg, int& ntiles) {
  dpg = a.dim / a.ngroups;
  tpg = (dpg + ssb::kCh - 1) / ssb::kCh;
  ntiles = (a.seqlen + ssb::kTile - 1) / ssb::kTile;
}

template <typename F>
int dispatch(int io, F&& f) {
  switch (io) {
    case SS_F32: return cuda_status(f(float{}));
    case SS_BF16: return cuda_status(f(__nv_bfloat16{}));
    case SS_F16: return cuda_status(f(__half{}));
    default: return SS_ERR_UNSUPPORTED;
  }
}

}  // namespace

extern "C" {

size_t ss_ckpt_elems(int batch, int dim, int seqlen, int dstate) {
  if (batch <= 0 || dim <= 0 || seqlen <= 0 || dstate <= 0) return 0;
  const size_t ntiles = ((size_t)seqlen + ssb::kTile - 1) / ssb::kTile;
  return (size_t)batch * ntiles * (size_t)dstate * (size_t)dim;
}

int ss_fwd(const ss_fwd_args* args, void* stream) {
  int rc = check_fwd(args);
  if (rc != SS_OK) return rc;
  if (!args->out || (args->out_batch_stride < 0 || args->out_dim_stride < 0)) return SS_ERR_INVALID;
  if (args->batch == 0 || args->seqlen == 0) return SS_OK;
  ssb::FwdK P{};
  P.a = *args;
  derive(P.a, P.dpg, P.tpg, P.ntiles);
  const size_t es = esize(args->io_dtype);
  P.vec_u = rows16(args->u, args->u_batch_stride, args->u_dim_stride, es);
  P.vec_d = rows16(args->delta, args->delta_batch_stride, args->delta_dim_stride, es);
  P.vec_z = args->z ? rows16(args->z, args->z_batch_stride, args->z_dim_stride, es) : 0;
  P.vec_out = rows16(args->out, args->out_batch_stride, args->out_dim_stride, es);
  cudaStream_t st = (cudaStream_t)stream;
  return dispatch(args->io_dtype, [&](auto tag) { return ssb::launch_fwd<decltype(tag)>(P, st); });
}

int ss_bwd(const ss_bwd_args* args, void* stream) {
  if (args == nullptr) return SS_ERR_INVALID;
  const ss_fwd_args& f = args->f;
  int rc = check_fwd(&f);
  if (rc != SS_OK) return rc;
  if (!args->dout || !args->du || !args->ddelta || !args->dA || !args->dB || !args->dC) return SS_ERR_INVALID;
  if (f.z && !args->dz) return SS_ERR_INVALID;
  if (!f.ckpt && f.seqlen > ssb::kTile && f.batch > 0) return SS_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  // accumulated outputs start from zero
  const size_t nA = (size_t)f.dim * f.dstate;
  const size_t nBv = (size_t)f.batch * f.ngroups * f.dstate * (size_t)f.seqlen;
  const size_t nB = f.var_B ? nBv : nA, nC = f.var_C ? nBv : nA;
  cudaError_t e = cudaMemsetAsync(args->dA, 0, nA * sizeof(float), st);
  if (e == cudaSuccess && nB) e = cudaMemsetAsync(args->dB, 0, nB * sizeof(float), st);
  if (e == cudaSuccess && nC) e = cudaMemsetAsync(args->dC, 0, nC * sizeof(float), st);
  if (e == cudaSuccess && args->dD) e = cudaMemsetAsync(args->dD, 0, (size_t)f.dim * sizeof(float), st);
  if (e == cudaSuccess && args->ddelta_bias)
    e = cudaMemsetAsync(args->ddelta_bias, 0, (size_t)f.dim * sizeof(float), st);
  if (e != cudaSuccess) return cuda_status(e);
  if (f.batch == 0 || f.seqlen == 0) return SS_OK;
  ssb::BwdK P{};
  P.a = *args;
  derive(f, P.dpg, P.tpg, P.ntiles);
  const size_t es = esize(f.io_dtype);
  P.vec_u = rows16(f.u, f.u_batch_stride, f.u_dim_stride, es);
  P.vec_d = rows16(f.delta, f.delta_batch_stride, f.delta_dim_stride, es);
  P.vec_z = f.z ? rows16(f.z, f.z_batch_stride, f.z_dim_stride, es) : 0;
  P.vec_dout = rows16(args->dout, args->dout_batch_stride, args->dout_dim_stride, es);
  P.vec_du = rows16(args->du, args->du_batch_stride, args->du_dim_stride, es);
  P.vec_dd = rows16(args->ddelta, args->ddelta_batch_stride, args->ddelta_dim_stride, es);
  P.vec_dz = f.z ? rows16(args->dz, args->dz_batch_stride, args->dz_dim_stride, es) : 0;
  P.vec_dbc = (f.seqlen % 4) == 0 && (reinterpret_cast<uintptr_t>(args->dB) & 15) == 0 &&
              (reinterpret_cast<uintptr_t>(args->dC) & 15) == 0;
  return dispatch(f.io_dtype, [&](auto tag) { return ssb::launch_bwd<decltype(tag)>(P, st); });
}

int ss_step(const ss_step_args* a, void* stream) {
  if (a == nullptr) return SS_ERR_INVALID;
  if (a->batch < 0 || a->dim < 1 || a->dstate < 1 || a->ngroups < 1 || a->dim % a->ngroups) return SS_ERR_INVALID;
  if (a->dstate > SS_MAX_DSTATE || a->batch > 65535) return SS_ERR_UNSUPPORTED;
  if (!dtype_ok(a->io_dtype) || !dtype_ok(a->bc_dtype)) return SS_ERR_UNSUPPORTED;
  if (a->bc_dtype != SS_F32 && a->bc_dtype != a->io_dtype) return SS_ERR_UNSUPPORTED;
  if (!a->state || !a->x || !a->dt || !a->A || !a->B || !a->C || !a->out) return SS_ERR_INVALID;
  if (a->batch == 0) return SS_OK;
  cudaStream_t st = (cudaStream_t)stream;
  return dispatch(a->io_dtype, [&](auto tag) { return ssb::launch_step<decltype(tag)>(*a, st); });
}

const char* ss_status_string(int s) {
  switch (s) {
    case SS_OK: return "ok";
    case SS_ERR_INVALID: return "invalid argument (null pointer, size, stride or group count)";
    case SS_ERR_UNSUPPORTED: return "unsupported dtype combination, dstate > 16 or batch > 65535";
    case SS_ERR_CUDA: return "CUDA runtime error (see ss_last_cuda_error)";
    default: return "unknown status";
  }
}

int ss_last_cuda_error(void) { return g_last_cuda; }

int ss_abi_version(void) { return SS_ABI_VERSION; }

size_t ss_struct_size(int which) {
  switch (which) {
    case 0: return sizeof(ss_fwd_args);
    case 1: return sizeof(ss_bwd_args);
    case 2: return sizeof(ss_step_args);
    default: return 0;
  }
}

}  // extern "C"
