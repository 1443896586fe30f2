/* CPU restatement of the reference selective scan (nmquan1503/Mamba,
 * csrc/selective_scan/forward_kernel.cu and backward_kernel.cu), plus the z gate of
 * modules/mamba_simple.py:143-146 and a single-token step.
 *
 * TEST INFRASTRUCTURE ONLY.  It is the parity checker for tests/, the CPU baseline
 * for bench.py, and nothing else: the mamba_b200 product never loads it.
 *
 * Two instantiations of ss_oracle_impl.h:
 *   *_f64 : double-precision state and sums — the parity oracle.
 *   *_f32 : float arithmetic like the reference kernels — the timed CPU baseline.
 * Both take fp32 tensors (bf16 inputs are widened by the caller).
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <omp.h>

#define REAL double
#define SUFFIX f64
#define EXP_(x) exp(x)
#define LOG1P_(x) log1p(x)
#include "ss_oracle_impl.h"
#undef REAL
#undef SUFFIX
#undef EXP_
#undef LOG1P_

#define REAL float
#define SUFFIX f32
#define EXP_(x) expf(x)
#define LOG1P_(x) log1pf(x)
#include "ss_oracle_impl.h"
#undef REAL
#undef SUFFIX
#undef EXP_
#undef LOG1P_

int ssor_max_threads(void) { return omp_get_max_threads(); }
