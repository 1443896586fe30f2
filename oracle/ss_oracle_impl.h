/* Body of the CPU restatement of the reference selective scan.  Included twice by
 * ss_oracle.c, once with REAL=double (the parity oracle) and once with REAL=float
 * (the timed CPU baseline).  TEST INFRASTRUCTURE ONLY: the product never links this.
 *
 * Layouts (all C-contiguous):
 *   u, delta, z, dout, out, du, ddelta, dz : (batch, dim, seqlen)
 *   A                                      : (dim, dstate)
 *   B, C variable                          : (batch, ngroups, dstate, seqlen)
 *   B, C constant                          : (dim, dstate)
 *   D, delta_bias, dD, ddelta_bias         : (dim)
 *   last_state                             : (batch, dim, dstate)
 *   state (step)                           : (batch, dim, dstate)
 */

#define CAT2(a, b) a##b
#define CAT(a, b) CAT2(a, b)
#define FN(name) CAT(name, SUFFIX)

/* delta' = softplus(delta + bias) with the reference's threshold of 20:
 * forward_kernel.cu:216-221 (delta + bias, then log1p(exp(.)) only when <= 20). */
static inline REAL FN(ssor_dt_)(REAL v, int softplus) {
    if (!softplus) return v;
    return v <= (REAL)20 ? LOG1P_(EXP_(v)) : v;
}

static inline REAL FN(ssor_sigmoid_)(REAL v) { return (REAL)1 / ((REAL)1 + EXP_(-v)); }

/* Forward over one (batch b, channel c) row.  Follows forward_kernel.cu:213-293:
 *   dA = exp(delta' * A[c,n])      (:228, :264 — exp2f(delta' * A * log2e))
 *   dBu = delta' * u * B[n,t]      (:222, :265)
 *   h   = dA * h + dBu             (ScanOp, common.h:70-82)
 *   y   = D * u + sum_n C[n,t] * h (:223, :287-293)
 * and then the gate y * silu(z) of modules/mamba_simple.py:143-146.
 * hist (nullable) receives h after every step, (seqlen, dstate). */
static void FN(ssor_fwd_row_)(int dim, int seqlen, int dstate, int ngroups, int var_B, int var_C,
                              int b, int c, const float* u, const float* delta, const float* A,
                              const float* B, const float* C, const float* D, const float* z,
                              const float* delta_bias, int softplus, const REAL* h0,
                              float* out, float* out_y, float* last_state, REAL* hist,
                              REAL* ahist, float* yloc) {
    const size_t row = ((size_t)b * dim + c) * (size_t)seqlen;
    const int dpg = dim / ngroups;
    const int g = c / dpg;
    const float* Bv = var_B ? B + ((size_t)b * ngroups + g) * (size_t)dstate * seqlen : B + (size_t)c * dstate;
    const float* Cv = var_C ? C + ((size_t)b * ngroups + g) * (size_t)dstate * seqlen : C + (size_t)c * dstate;
    const REAL Dc = D ? (REAL)D[c] : (REAL)0;
    const REAL bias = delta_bias ? (REAL)delta_bias[c] : (REAL)0;
    REAL h[256];
    for (int n = 0; n < dstate; n++) h[n] = h0 ? h0[n] : (REAL)0;
    for (int t = 0; t < seqlen; t++) {
        const REAL uv = (REAL)u[row + t];
        const REAL dt = FN(ssor_dt_)((REAL)delta[row + t] + bias, softplus);
        REAL y = Dc * uv;
        for (int n = 0; n < dstate; n++) {
            const REAL a = EXP_(dt * (REAL)A[(size_t)c * dstate + n]);
            const REAL bn = var_B ? (REAL)Bv[(size_t)n * seqlen + t] : (REAL)Bv[n];
            const REAL cn = var_C ? (REAL)Cv[(size_t)n * seqlen + t] : (REAL)Cv[n];
            h[n] = a * h[n] + dt * uv * bn;
            y += cn * h[n];
            if (hist) hist[(size_t)t * dstate + n] = h[n];
            if (ahist) ahist[(size_t)t * dstate + n] = a;
        }
        if (out_y) out_y[row + t] = (float)y;
        if (yloc) yloc[t] = (float)y;
        if (z) {
            const REAL zv = (REAL)z[row + t];
            y = y * zv * FN(ssor_sigmoid_)(zv);
        }
        if (out) out[row + t] = (float)y;
    }
    if (last_state)
        for (int n = 0; n < dstate; n++)
            last_state[((size_t)b * dim + c) * dstate + n] = (float)h[n];
}

int FN(ssor_fwd_)(int batch, int dim, int seqlen, int dstate, int ngroups, int var_B, int var_C,
                  const float* u, const float* delta, const float* A, const float* B, const float* C,
                  const float* D, const float* z, const float* delta_bias, int softplus,
                  const float* h0, float* out, float* out_y, float* last_state, int nthreads) {
    if (dstate > 256 || dstate < 1 || ngroups < 1 || dim % ngroups) return 1;
    if (nthreads > 0) omp_set_num_threads(nthreads);
    const long rows = (long)batch * dim;
#pragma omp parallel for schedule(dynamic, 4)
    for (long r = 0; r < rows; r++) {
        const int b = (int)(r / dim), c = (int)(r % dim);
        REAL h0r[256];
        if (h0)
            for (int n = 0; n < dstate; n++) h0r[n] = (REAL)h0[r * dstate + n];
        FN(ssor_fwd_row_)(dim, seqlen, dstate, ngroups, var_B, var_C, b, c, u, delta, A, B, C, D, z,
                          delta_bias, softplus, h0 ? h0r : NULL, out, out_y, last_state, NULL, NULL, NULL);
    }
    return 0;
}

/* Backward.  Follows backward_kernel.cu:
 *   dD      += dout * u                                   (:338-340)
 *   du       = D * dout + sum_n dh * B * delta'           (:334, :438)
 *   ddelta' += dh * B * u + dh * A * (h_t - dBu_t)        (:439-440)
 *   dA      += dh * delta' * (h_t - dBu_t)                (:441)
 *   dB[t]   += dh * delta' * u        (summed over channels of the group, :451, :466-478)
 *   dC[t]   += dout * h_t                                 (:454)
 *   ddelta   = ddelta' * sigmoid(delta + bias) where delta + bias <= 20 (:499-517)
 *   ddelta_bias += ddelta                                 (:519-521, :556-561)
 * where dh = dL/dh_t comes from the reverse recurrence dh_t = C_t dout_t + dA_{t+1} dh_{t+1}
 * (reverse_scan.cuh over (dA_{t+1}, C_t dout_t), :396-428).  With a gate z, the scan sees
 * dout * silu(z) and dz = dout * y * silu'(z) (the derivative of mamba_simple.py:143-146).
 * Constant (2-D) B / C produce (dim, dstate) gradients summed over batch and time (:563-585). */
int FN(ssor_bwd_)(int batch, int dim, int seqlen, int dstate, int ngroups, int var_B, int var_C,
                  const float* u, const float* delta, const float* A, const float* B, const float* C,
                  const float* D, const float* z, const float* delta_bias, int softplus,
                  const float* dout, float* du, float* ddelta, float* dA, float* dB, float* dC,
                  float* dD, float* dz, float* ddelta_bias, int nthreads) {
    if (dstate > 256 || dstate < 1 || ngroups < 1 || dim % ngroups) return 1;
    if (nthreads > 0) omp_set_num_threads(nthreads);
    const int dpg = dim / ngroups;
    const size_t nB = var_B ? (size_t)batch * ngroups * dstate * seqlen : (size_t)dim * dstate;
    const size_t nC = var_C ? (size_t)batch * ngroups * dstate * seqlen : (size_t)dim * dstate;
    int nt = 1;
#pragma omp parallel
    {
#pragma omp single
        nt = omp_get_num_threads();
    }
    REAL* accB = (REAL*)calloc((size_t)nt * nB, sizeof(REAL));
    REAL* accC = (REAL*)calloc((size_t)nt * nC, sizeof(REAL));
    REAL* accA = (REAL*)calloc((size_t)dim * dstate, sizeof(REAL));
    if (!accB || !accC || !accA) {
        free(accB); free(accC); free(accA);
        return 2;
    }
#pragma omp parallel num_threads(nt)
    {
        const int tid = omp_get_thread_num();
        REAL* myB = accB + (size_t)tid * nB;
        REAL* myC = accC + (size_t)tid * nC;
        REAL* hist = (REAL*)malloc((size_t)seqlen * dstate * sizeof(REAL));
        REAL* ahist = (REAL*)malloc((size_t)seqlen * dstate * sizeof(REAL));
        float* yrow = (float*)malloc((size_t)seqlen * sizeof(float));
        REAL dh[256], dAc[256];
#pragma omp for schedule(dynamic, 1)
        for (int c = 0; c < dim; c++) {
            const int g = c / dpg;
            const REAL Dc = D ? (REAL)D[c] : (REAL)0;
            const REAL bias = delta_bias ? (REAL)delta_bias[c] : (REAL)0;
            REAL dDc = 0, dbc = 0;
            for (int n = 0; n < dstate; n++) dAc[n] = 0;
            for (int b = 0; b < batch; b++) {
                const size_t row = ((size_t)b * dim + c) * (size_t)seqlen;
                const float* Bv = var_B ? B + ((size_t)b * ngroups + g) * (size_t)dstate * seqlen : B + (size_t)c * dstate;
                const float* Cv = var_C ? C + ((size_t)b * ngroups + g) * (size_t)dstate * seqlen : C + (size_t)c * dstate;
                REAL* dBv = var_B ? myB + ((size_t)b * ngroups + g) * (size_t)dstate * seqlen : myB + (size_t)c * dstate;
                REAL* dCv = var_C ? myC + ((size_t)b * ngroups + g) * (size_t)dstate * seqlen : myC + (size_t)c * dstate;
                /* recompute the forward states (the reference recomputes from its chunk carry x) */
                FN(ssor_fwd_row_)(dim, seqlen, dstate, ngroups, var_B, var_C, b, c, u, delta, A, B, C, D,
                                  NULL, delta_bias, softplus, NULL, NULL, NULL, NULL, hist, ahist, yrow);
                for (int n = 0; n < dstate; n++) dh[n] = 0;
                for (int t = seqlen - 1; t >= 0; t--) {
                    const REAL uv = (REAL)u[row + t];
                    const REAL v = (REAL)delta[row + t] + bias;
                    const REAL dt = FN(ssor_dt_)(v, softplus);
                    REAL dy = (REAL)dout[row + t];
                    if (z) {
                        const REAL zv = (REAL)z[row + t];
                        const REAL s = FN(ssor_sigmoid_)(zv);
                        if (dz) dz[row + t] = (float)(dy * (REAL)yrow[t] * s * ((REAL)1 + zv * ((REAL)1 - s)));
                        dy = dy * zv * s;
                    }
                    REAL dut = Dc * dy, ddt = 0;
                    dDc += dy * uv;
                    for (int n = 0; n < dstate; n++) {
                        const REAL An = (REAL)A[(size_t)c * dstate + n];
                        const REAL bn = var_B ? (REAL)Bv[(size_t)n * seqlen + t] : (REAL)Bv[n];
                        const REAL cn = var_C ? (REAL)Cv[(size_t)n * seqlen + t] : (REAL)Cv[n];
                        const REAL anext = (t + 1 < seqlen) ? ahist[(size_t)(t + 1) * dstate + n] : (REAL)0;
                        dh[n] = cn * dy + anext * dh[n];
                        const REAL a = ahist[(size_t)t * dstate + n];
                        const REAL hprev = t > 0 ? hist[(size_t)(t - 1) * dstate + n] : (REAL)0;
                        const REAL ah = a * hprev;
                        dut += dh[n] * bn * dt;
                        ddt += dh[n] * (bn * uv + An * ah);
                        dAc[n] += dh[n] * dt * ah;
                        if (var_B) dBv[(size_t)n * seqlen + t] += dh[n] * dt * uv;
                        else dBv[n] += dh[n] * dt * uv;
                        if (var_C) dCv[(size_t)n * seqlen + t] += dy * hist[(size_t)t * dstate + n];
                        else dCv[n] += dy * hist[(size_t)t * dstate + n];
                    }
                    if (softplus && v <= (REAL)20) ddt = ddt * FN(ssor_sigmoid_)(v);
                    du[row + t] = (float)dut;
                    ddelta[row + t] = (float)ddt;
                    dbc += ddt;
                }
            }
            for (int n = 0; n < dstate; n++) accA[(size_t)c * dstate + n] = dAc[n];
            if (dD) dD[c] = (float)dDc;
            if (ddelta_bias) ddelta_bias[c] = (float)dbc;
        }
        free(hist);
        free(ahist);
        free(yrow);
    }
    for (size_t i = 0; i < (size_t)dim * dstate; i++) dA[i] = (float)accA[i];
#pragma omp parallel for
    for (long i = 0; i < (long)nB; i++) {
        REAL s = 0;
        for (int t = 0; t < nt; t++) s += accB[(size_t)t * nB + i];
        dB[i] = (float)s;
    }
#pragma omp parallel for
    for (long i = 0; i < (long)nC; i++) {
        REAL s = 0;
        for (int t = 0; t < nt; t++) s += accC[(size_t)t * nC + i];
        dC[i] = (float)s;
    }
    free(accB); free(accC); free(accA);
    return 0;
}

/* Single-token state update: one step of the forward recurrence above from a given state,
 * h <- exp(dt*A) h + dt*B*x, y = C.h + D x, y *= silu(z).  The reference has no step
 * function (models/causal_lm.py:61-62 is a stub); this is the forward at seqlen 1
 * with an initial state, which is how the decode path is pinned. */
int FN(ssor_step_)(int batch, int dim, int dstate, int ngroups, float* state, const float* x,
                   const float* dt, const float* A, const float* B, const float* C, const float* D,
                   const float* z, const float* dt_bias, int softplus, float* out) {
    if (dstate > 256 || dim % ngroups) return 1;
    const int dpg = dim / ngroups;
    for (int b = 0; b < batch; b++)
        for (int c = 0; c < dim; c++) {
            const int g = c / dpg;
            const size_t r = (size_t)b * dim + c;
            const REAL xv = (REAL)x[r];
            const REAL d = FN(ssor_dt_)((REAL)dt[r] + (dt_bias ? (REAL)dt_bias[c] : (REAL)0), softplus);
            REAL y = D ? (REAL)D[c] * xv : (REAL)0;
            for (int n = 0; n < dstate; n++) {
                const size_t si = r * dstate + n;
                const size_t bi = ((size_t)b * ngroups + g) * dstate + n;
                const REAL a = EXP_(d * (REAL)A[(size_t)c * dstate + n]);
                const REAL h = a * (REAL)state[si] + d * xv * (REAL)B[bi];
                state[si] = (float)h;
                y += (REAL)C[bi] * h;
            }
            if (z) y = y * (REAL)z[r] * FN(ssor_sigmoid_)((REAL)z[r]);
            out[r] = (float)y;
        }
    return 0;
}

#undef FN
#undef CAT
#undef CAT2
