/*
 * mamba_b200 selective scan — C ABI of libmamba_b200_ss.so (sm_100a).
 *
 * Plain pointers and sizes only.  Every call is asynchronous on the given CUDA stream
 * (a cudaStream_t passed as void*; NULL = legacy default stream) and returns an
 * ss_status.  Device pointers must belong to the current device.
 *
 * Reference interfaces these entry points replace (nmquan1503/Mamba):
 *   ss_fwd  <- selective_scan.forward(u, delta, A, B, C, D?, delta_bias?, use_delta_softplus)
 *              -> [out, x]          csrc/selective_scan/selective_scan.cpp:184-244, :331-334
 *              (kernel launcher forward_kernel_launch, forward_kernel.cu:313-333)
 *   ss_bwd  <- selective_scan.backward(u, delta, A, B, C, D?, delta_bias?, dout, x?, flag)
 *              -> [du, ddelta, dA, dB, dC, dD, ddelta_bias]
 *                                   csrc/selective_scan/selective_scan.cpp:246-329, :331-334
 *              (kernel launcher backward_kernel_launch, backward_kernel.cu:588-618)
 *   ss_step <- no counterpart: the reference has no decode step (models/causal_lm.py:61-62
 *              is a stub).  It is one step of the same recurrence from a stored state.
 *   ss_conv_fwd / ss_conv_bwd <- the input side of the reference's MambaSimple.forward,
 *              modules/mamba_simple.py:91-98 (input_proj output -> permute(0,2,1).contiguous()
 *              -> chunk -> short_conv (nn.Conv1d depthwise, padding width-1, cut to seqlen,
 *              :41-48) -> SiLU), which the reference runs as separate PyTorch kernels with
 *              copies; here one pass reads the projection's (batch, seqlen, dim) layout
 *              directly and writes the scan's (batch, dim, seqlen) layout.
 *   ss_conv_step <- no counterpart (no decode in the reference): the same convolution for
 *              one new input from a rolling state of the previous width-1 inputs.
 *   ss_mamba_step <- no counterpart: one decode step of a MambaSimple block's mixer (conv step,
 *              x projection, delta projection, SSM step, gate; modules/mamba_simple.py:93-146
 *              for one token) in one kernel.
 *   ss_rmsnorm_fwd / ss_rmsnorm_bwd <- the reference's RMSNorm.forward (modules/rms_norm.py:
 *              21-30) fused with its Block's residual add (models/causal_lm.py:30-37), which
 *              the reference runs as a chain of PyTorch elementwise and reduction kernels.
 *
 * Tensor layouts (element strides; the innermost sequence axis must have stride 1, or, with
 * ss_fwd_args.layout = SS_LAYOUT_BLD, the innermost dim axis):
 *   u, delta, z, out, dout, du, ddelta, dz : (batch, dim, seqlen), batch/dim strides given
 *   A, dA                                  : (dim, dstate) contiguous, fp32
 *   B, C   variable                        : (batch, ngroups, dstate, seqlen) contiguous
 *   B, C   constant                        : (dim, dstate) contiguous
 *   dB, dC                                 : same shape as B, C, always fp32
 *   D, delta_bias, dD, ddelta_bias         : (dim) fp32
 *   ckpt                                   : opaque fp32 buffer of ss_ckpt_elems() floats;
 *                                            written by ss_fwd, read by ss_bwd
 *   out_y, y                               : (batch, dim, seqlen) ungated output, I/O dtype
 *   last_state                             : (batch, dim, dstate) fp32
 * Channel c uses group c / (dim / ngroups), as forward_kernel.cu:144 of the reference.
 */
#ifndef MAMBA_B200_SS_H
#define MAMBA_B200_SS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SS_ABI_VERSION 8
/* the reference's kernels dispatch dstate up to 256 (csrc/selective_scan/static_switch.h:15-35) */
#define SS_MAX_DSTATE 256
#define SS_MAX_CONV_WIDTH 4
/* capacity (floats) of the library-held state array used by ss_bwd_noalloc: 16 MiB */
#define SS_NOALLOC_MAX_CKPT_ELEMS 4194304

#if defined(__GNUC__)
#define SS_API __attribute__((visibility("default")))
#else
#define SS_API
#endif

typedef enum ss_dtype { SS_F32 = 0, SS_BF16 = 1, SS_F16 = 2 } ss_dtype;

/* Layout of the per-element tensors of a scan call (u, delta, z, out, out_y and, in the
 * backward, dout, du, ddelta, dz, y):
 *   SS_LAYOUT_BDL  (batch, dim, seqlen) with unit seqlen stride (the reference's layout);
 *   SS_LAYOUT_BLD  (batch, seqlen, dim) with unit dim stride — the layout of the projections
 *                  around the scan in a Mamba block (modules/mamba_simple.py:96, :104-106,
 *                  :143-145 permute to and from it); every *_dim_stride field of the call then
 *                  holds the stride between consecutive time steps.
 * SS_LAYOUT_BLD needs dstate <= 16 and 16-byte aligned rows (tensor maps); otherwise the call
 * returns SS_ERR_UNSUPPORTED. */
typedef enum ss_layout { SS_LAYOUT_BDL = 0, SS_LAYOUT_BLD = 1 } ss_layout;

typedef enum ss_status {
  SS_OK = 0,
  SS_ERR_INVALID = 1,     /* null pointer, bad size, bad stride, dim % ngroups != 0 */
  SS_ERR_UNSUPPORTED = 2, /* dtype combination, dstate > SS_MAX_DSTATE or a size the grid cannot hold */
  SS_ERR_CUDA = 3         /* a CUDA runtime call or kernel launch failed */
} ss_status;

typedef struct ss_fwd_args {
  int batch, dim, seqlen, dstate, ngroups;
  int var_B, var_C;         /* 1: (batch, ngroups, dstate, seqlen); 0: (dim, dstate)      */
  int delta_softplus;       /* delta' = softplus(delta + delta_bias), threshold 20        */
  int io_dtype;             /* ss_dtype of u, delta, z, out                               */
  int bc_dtype;             /* ss_dtype of B, C: SS_F32 or io_dtype                       */
  const void* u;     int64_t u_batch_stride, u_dim_stride;
  const void* delta; int64_t delta_batch_stride, delta_dim_stride;
  const float* A;
  const void* B;
  const void* C;
  const float* D;           /* nullable: D = 0                                            */
  const void* z;     int64_t z_batch_stride, z_dim_stride;  /* nullable: no gate          */
  const float* delta_bias;  /* nullable: bias = 0                                         */
  void* out;         int64_t out_batch_stride, out_dim_stride; /* y or y * silu(z)        */
  float* ckpt;              /* nullable: skip the states the backward needs               */
  float* last_state;        /* nullable; zeros when seqlen == 0 (the zero initial state)  */
  void* out_y;       int64_t out_y_batch_stride, out_y_dim_stride;
                            /* nullable: the ungated y (D*u + C.h), which ss_bwd needs when
                               z is given; written only when z is given                   */
  float* work;              /* 16-byte aligned fp32 scratch of ss_work_elems(batch, dim,
                               seqlen, dstate) floats, required when that is > 0 (dstate > 16: the states
                               are scanned in groups of 16 whose per-element sums meet
                               here); ss_fwd and ss_bwd overwrite it; contents are not
                               needed between calls.  Nullable when dstate <= 16.          */
  int layout;               /* ss_layout of the per-element tensors (0: batch, dim, seqlen)  */
} ss_fwd_args;

typedef struct ss_bwd_args {
  ss_fwd_args f;            /* the forward's inputs; f.out, f.last_state are ignored;
                               f.ckpt must hold what ss_fwd wrote for the same inputs     */
  const void* dout;  int64_t dout_batch_stride, dout_dim_stride;
  void* du;          int64_t du_batch_stride, du_dim_stride;
  void* ddelta;      int64_t ddelta_batch_stride, ddelta_dim_stride;
  void* dz;          int64_t dz_batch_stride, dz_dim_stride;   /* required iff f.z       */
  const void* y;     int64_t y_batch_stride, y_dim_stride;     /* required iff f.z: the
                               forward's out_y (may alias dz: each element of y is read
                               before the same element of dz is written)                 */
  float* dA;                /* overwritten (zeroed, then accumulated)                     */
  float* dB;                /* overwritten                                                */
  float* dC;                /* overwritten                                                */
  float* dD;                /* nullable; overwritten                                      */
  float* ddelta_bias;       /* nullable; overwritten                                      */
} ss_bwd_args;

typedef struct ss_step_args {
  int batch, dim, dstate, ngroups;
  int dt_softplus;
  int io_dtype;             /* dtype of x, dt, z, out, dt_proj                            */
  int bc_dtype;             /* dtype of B, C: SS_F32 or io_dtype                          */
  float* state;      int64_t state_batch_stride;  /* (batch, dim, dstate) fp32, in/out    */
  const void* x;     int64_t x_batch_stride;      /* (batch, dim)                         */
  const void* dt;    int64_t dt_batch_stride;     /* (batch, dim); (batch, dt_rank) with dt_proj */
  const float* A;                                 /* (dim, dstate)                        */
  const void* B;     int64_t B_batch_stride;      /* (batch, ngroups, dstate), groups and
                                                     states packed; batch stride in
                                                     elements, 0 = packed                 */
  const void* C;     int64_t C_batch_stride;
  const float* D;                                 /* nullable                             */
  const void* z;     int64_t z_batch_stride;      /* nullable                             */
  const float* dt_bias;                           /* nullable                             */
  void* out;         int64_t out_batch_stride;    /* (batch, dim)                         */
  const void* dt_proj; int dt_rank;               /* nullable: dt = dt_in . dt_proj[c, :], dt_proj
                                                     (dim, dt_rank) row-major, dt_rank <= 1024
                                                     (the delta projection, fused)          */
} ss_step_args;

/* Causal depthwise convolution (+ SiLU) of the (batch, seqlen, dim) input x into the scan's
 * (batch, dim, seqlen) layout:
 *   pre[b,c,t] = bias[c] + sum_{k<width} weight[c,k] * x[b, t-(width-1)+k, c]
 *   u[b,c,t]   = silu ? pre * sigmoid(pre) : pre
 * x at t < 0 is state_in[b, c, t + width-1] (oldest first) or zero when state_in is NULL (the
 * reference's zero padding).  z, when given, is copied from (batch, seqlen, dim) to zt
 * (batch, dim, seqlen) in the same pass.  state_out, when given, receives the last width-1
 * inputs (for a following chunk or ss_conv_step); it must not alias state_in.  ss_conv_fwd and
 * ss_conv_bwd use state_in entries at the I/O precision (exact for states this library wrote,
 * which are earlier inputs of the same dtype); ss_conv_step keeps them in fp32. */
typedef struct ss_conv_args {
  int batch, dim, seqlen, width; /* width 1..SS_MAX_CONV_WIDTH                              */
  int silu;                      /* apply SiLU                                              */
  int io_dtype;                  /* dtype of x, z, u, zt                                    */
  const void* x;     int64_t x_batch_stride, x_seq_stride;   /* (batch, seqlen, dim), dim stride 1 */
  const float* weight;           /* (dim, width) fp32 contiguous                            */
  const float* bias;             /* (dim) fp32, nullable                                    */
  const float* state_in;         /* (batch, dim, width-1) fp32 contiguous, nullable        */
  float* state_out;              /* (batch, dim, width-1) fp32 contiguous, nullable        */
  void* u;           int64_t u_batch_stride, u_dim_stride;   /* (batch, dim, seqlen), seq stride 1 */
  const void* z;     int64_t z_batch_stride, z_seq_stride;   /* nullable (batch, seqlen, dim)      */
  void* zt;          int64_t zt_batch_stride, zt_dim_stride; /* (batch, dim, seqlen); iff z        */
} ss_conv_args;

/* Backward of ss_conv_fwd: from du (gradient of u) it writes dx in the (batch, seqlen, dim)
 * layout and overwrites dweight / dbias; dzt, when given, is copied transposed into dz (the
 * gate half of the projection's gradient).  f holds the forward's arguments (x, weight,
 * bias, state_in, silu; its u / z / zt / state_out are ignored). */
typedef struct ss_conv_bwd_args {
  ss_conv_args f;
  const void* du;    int64_t du_batch_stride, du_dim_stride;   /* (batch, dim, seqlen)        */
  void* dx;          int64_t dx_batch_stride, dx_seq_stride;   /* (batch, seqlen, dim)        */
  const void* dzt;   int64_t dzt_batch_stride, dzt_dim_stride; /* nullable (batch, dim, seqlen) */
  void* dz;          int64_t dz_batch_stride, dz_seq_stride;   /* (batch, seqlen, dim); iff dzt */
  float* dweight;    /* (dim, width) fp32, overwritten                                      */
  float* dbias;      /* (dim) fp32, nullable, overwritten                                   */
} ss_conv_bwd_args;

/* One decode step of the convolution: window = [state (oldest first), x];
 * u = silu(bias + weight . window); state <- window[1:]. */
typedef struct ss_conv_step_args {
  int batch, dim, width, silu, io_dtype;
  float* state;      int64_t state_batch_stride;  /* (batch, dim, width-1) fp32, in/out      */
  const void* x;     int64_t x_batch_stride;      /* (batch, dim)                           */
  const float* weight;                            /* (dim, width) fp32                      */
  const float* bias;                              /* (dim) fp32, nullable                   */
  void* u;           int64_t u_batch_stride;      /* (batch, dim)                           */
} ss_conv_step_args;

/* Residual add + RMSNorm over rows of length dim (dim <= 2048 for 2-byte I/O, <= 1024 for fp32):
 *   h = x + residual   (rounded to the I/O dtype; h = x when residual is NULL)
 *   y = h * rsqrt(mean(h^2) + eps) * (unit_offset ? 1 + weight : weight)
 * residual_out (needs residual) receives h; rstd (rows, fp32) keeps rsqrt(mean(h^2) + eps)
 * for the backward.  The reference's RMSNorm is unit_offset = 1 (modules/rms_norm.py:29). */
typedef struct ss_rmsnorm_args {
  int rows, dim, io_dtype, unit_offset;
  float eps;
  const void* x;         int64_t x_row_stride;
  const void* residual;  int64_t residual_row_stride;       /* nullable                      */
  const float* weight;                                       /* (dim) fp32                    */
  void* y;               int64_t y_row_stride;
  void* residual_out;    int64_t residual_out_row_stride;   /* nullable                      */
  float* rstd;                                               /* (rows) fp32, nullable         */
} ss_rmsnorm_args;

/* Backward of ss_rmsnorm_fwd from dy: dh = d loss / d h (plus dh_in, the gradient already
 * flowing into h through the residual stream, when given) — also the gradient of x and of
 * residual — and dweight (overwritten).  h is the normalised input (residual_out, or x). */
typedef struct ss_rmsnorm_bwd_args {
  int rows, dim, io_dtype, unit_offset;
  const void* h;         int64_t h_row_stride;
  const float* weight;                                       /* (dim) fp32                    */
  const float* rstd;                                         /* (rows) fp32 from the forward  */
  const void* dy;        int64_t dy_row_stride;
  const void* dh_in;     int64_t dh_in_row_stride;          /* nullable                      */
  void* dh;              int64_t dh_row_stride;
  float* dweight;                                            /* (dim) fp32, overwritten       */
} ss_rmsnorm_bwd_args;

/* One decode step of a Mamba block's mixer, between its input and output projections:
 *   x, z = xz[b, :dim], xz[b, dim:]
 *   u    = silu(conv_bias + conv_weight . [conv_state, x]);  conv_state rolls in
 *   dbl  = x_proj u  (dt_rank + 2 dstate values: dt_in, B, C)
 *   dt   = dt_proj dt_in + dt_bias  (softplus'd when dt_softplus)
 *   ssm_state = exp(dt A) ssm_state + dt u B;   y = (C . ssm_state + D u) * silu(z)
 * u and dbl are rounded to the I/O dtype (as the stored activations of the prompt path). */
typedef struct ss_mamba_step_args {
  int batch, dim, dstate, width, dt_rank, io_dtype, dt_softplus;
  const void* xz;        int64_t xz_batch_stride;   /* (batch, 2 dim), unit stride along dim  */
  float* conv_state;                                 /* (batch, dim, width-1) fp32, packed     */
  const float* conv_weight;                          /* (dim, width) fp32                      */
  const float* conv_bias;                            /* (dim) fp32, nullable                   */
  const void* x_proj;                                /* (dt_rank + 2 dstate, dim) row-major    */
  const void* dt_proj;                               /* (dim, dt_rank) row-major               */
  const float* dt_bias;                              /* (dim) fp32, nullable                   */
  const float* A;                                    /* (dim, dstate) fp32                     */
  const float* D;                                    /* (dim) fp32, nullable                   */
  float* ssm_state;                                  /* (batch, dim, dstate) fp32, packed      */
  void* y;               int64_t y_batch_stride;    /* (batch, dim): the gated output         */
} ss_mamba_step_args;

/* Number of fp32 elements of the forward-to-backward state buffer. */
SS_API size_t ss_ckpt_elems(int batch, int dim, int seqlen, int dstate);

/* Number of fp32 elements of the scratch ss_fwd_args.work holds.  dstate > 16: 2 * batch * dim *
 * seqlen (ss_fwd uses the first half, ss_bwd all of it; required).  dstate <= 16: 0 when one
 * CTA per (batch row, 32 channels) fills the GPU, else batch * K * (dstate + 1) * dim for the
 * K time chunks the sequence is cut into (a summary per chunk); optional — a call without it
 * scans each row in one piece.  Size it after any ss_set_time_chunks call. */
SS_API size_t ss_work_elems(int batch, int dim, int seqlen, int dstate);

/* Forward scan: out = (D*u + sum_n C*h) [* silu(z)], h_t = exp(delta'*A) h_{t-1} + delta'*u*B.
 * With time chunks (see ss_work_elems) it runs a summary pass over the chunks, then the main pass
 * as a programmatic dependent of it; the backward does the same with its carry pass. */
SS_API int ss_fwd(const ss_fwd_args* args, void* stream);

/* Backward scan: all input gradients from dout, using the forward's ckpt.  On `stream` it runs a
 * kernel that zeroes dA / dB / dC / dD / ddelta_bias (one span per run of buffers that lie end to
 * end, so callers may allocate them adjacently to save launches), then the backward, launched as
 * a programmatic dependent that may start before the zeroing ends and waits for it before
 * accumulating (dstate > 16: memsets and an ordinary launch). */
SS_API int ss_bwd(const ss_bwd_args* args, void* stream);

/* Backward scan for callers that cannot allocate device memory (an FFI host without a
 * CUDA allocator, a process whose device memory belongs to its own pool, any caller for
 * which a cudaMalloc mid-step would fail or synchronise the device).  No counterpart in
 * the reference.  It ignores args->f.ckpt: it recomputes the forward states into a
 * state array held by the library (one per GPU that loads it, kept until exit) and runs
 * the backward from there, calling no allocator.  Limits: ss_ckpt_elems(...) of the call
 * must be <= SS_NOALLOC_MAX_CKPT_ELEMS, else SS_ERR_UNSUPPORTED.  Every argument is checked
 * before anything is launched.  The first call on a device (and the first after its CUDA
 * context changes) looks up that array's address: make it before any stream capture.  All calls
 * on a device share the array: calls that overlap on the GPU race.  du (and dz, with a gate)
 * receive the recomputed forward outputs before the backward overwrites them, so they must
 * not alias an input; args->y is ignored.  With dstate > 16 the caller's args->f.work
 * (ss_work_elems floats) is required, as for ss_bwd. */
SS_API int ss_bwd_noalloc(const ss_bwd_args* args, void* stream);

/* One decode step: state <- exp(dt'*A) state + dt'*x*B; out = (C.state + D x) [* silu(z)],
 * dt' = softplus(dt + dt_bias) when dt_softplus; with dt_proj, dt is first projected from the
 * dt_rank inputs (the reference block's delta_proj, modules/mamba_simple.py:56-60, :114). */
SS_API int ss_step(const ss_step_args* args, void* stream);

/* Convolution + SiLU on the input side of a Mamba block (see ss_conv_args). */
SS_API int ss_conv_fwd(const ss_conv_args* args, void* stream);

/* Its backward (see ss_conv_bwd_args). */
SS_API int ss_conv_bwd(const ss_conv_bwd_args* args, void* stream);

/* One decode step of the convolution (see ss_conv_step_args). */
SS_API int ss_conv_step(const ss_conv_step_args* args, void* stream);

/* One decode step of a block's mixer (see ss_mamba_step_args). */
SS_API int ss_mamba_step(const ss_mamba_step_args* args, void* stream);

/* Residual add + RMSNorm (see ss_rmsnorm_args). */
SS_API int ss_rmsnorm_fwd(const ss_rmsnorm_args* args, void* stream);

/* Its backward (see ss_rmsnorm_bwd_args). */
SS_API int ss_rmsnorm_bwd(const ss_rmsnorm_bwd_args* args, void* stream);

/* Static description of a status code. */
SS_API const char* ss_status_string(int status);

/* The CUDA error (cudaError_t as int) behind the last SS_ERR_CUDA on this thread. */
SS_API int ss_last_cuda_error(void);

/* Error bits that kernels raised on the current device since the last reset (1: a bounded
 * wait for a TMA tile gave up), or -1 if the status cannot be read.  Synchronizes `stream`;
 * reset != 0 clears the bits. */
SS_API int ss_device_status(int reset, void* stream);

/* Limit, in SM clock cycles, of every bounded wait the scan kernels make for a TMA tile, for
 * the launches that follow from this process (all threads); returns the previous limit.
 * cycles < 0 restores the default (4e9 cycles, about 2 s).  A wait that runs out raises bit 1
 * of the device status (ss_device_status), lets the CTA's copies in flight land (bounded by
 * the default) and ends the CTA, leaving its outputs incomplete.  No counterpart in the
 * reference, whose kernels have no waits on memory copies. */
SS_API long long ss_set_wait_limit(long long cycles);

/* Time chunks per scan pass for the calls that follow from this process: 0 (the default)
 * chooses them from the shape, k >= 1 forces min(k, tiles of 16 steps) whenever a workspace of
 * ss_work_elems floats is given (1: never split).  Returns the previous setting.  A testing
 * and tuning knob; no counterpart in the reference. */
SS_API int ss_set_time_chunks(int chunks);

/* SS_ABI_VERSION of the loaded library. */
SS_API int ss_abi_version(void);

/* sizeof the argument structs as compiled into the library (0: ss_fwd_args,
 * 1: ss_bwd_args, 2: ss_step_args, 3: ss_conv_args, 4: ss_conv_bwd_args,
 * 5: ss_conv_step_args, 6: ss_rmsnorm_args, 7: ss_rmsnorm_bwd_args, 8: ss_mamba_step_args;
 * 0 for other values) — lets an FFI binding check its own struct
 * layout against the library's. */
SS_API size_t ss_struct_size(int which);

#ifdef __cplusplus
}
#endif

#endif /* MAMBA_B200_SS_H */
