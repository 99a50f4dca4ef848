/*
 * oracle_impl.h -- body of the CPU restatement, included twice by oracle.c:
 * once with REAL=double (the golden FP64 oracle) and once with REAL=float (a
 * sequential FP32 port of the reference recurrences, used as the timed CPU
 * baseline). TEST INFRASTRUCTURE ONLY: nothing in the product links this.
 *
 * Every function restates the reference kernel's arithmetic token by token.
 * Citations are to XMetAI-Lab/xmetai-onnx-plugins, paths within that project.
 */

#ifndef REAL
#error "define REAL before including oracle_impl.h"
#endif

/* ------------------------------------------------------------------ SelectiveScanFn
 * Per (batch b, channel d), with g = d / (dim / n_groups):
 *   delta_t = delta[b,d,t] + bias[d]; softplus when enabled
 *             (selective_scan_fwd_kernel.cuh:150-163: x <= 20 ? log1p(exp(x)) : x)
 *   out_t   = D[d] * u_t  (:161)
 *   for n:  h_n = exp(delta_t * A[d,n]) * h_n + delta_t * u_t * Bhat   (:166-237, scan op
 *           selective_scan_common.h:148-153 (a1*a0, a1*b0 + b1))
 *           out_t += Chat * h_n                                         (:258-268)
 *   Bhat = B[b,g,n,t] (variable B) or 1 (constant B folded into Chat, :179-210);
 *   Chat = C[b,g,n,t] (variable C) * B[d,n] when B is constant, C[d,n] when C is
 *   constant, B[d,n]*C[d,n] when both are constant.
 *   gate: out_t *= z_t / (1 + exp(-z_t))  (:283-301, the out_z buffer)
 * gb / gc: group count of a variable B / C ([batch, g, N, L]); 0 = constant [dim, N].
 */
static void FN(ss_unit)(int b, int d, int dim, int seqlen, int dstate, int gb, int gc,
                        const float *u, const float *delta, const float *A, const float *Bm,
                        const float *Cm, const float *Dv, const float *z, const float *bias,
                        int softplus, int gate, OUT_T *out, OUT_T *last) {
    const int n_groups = gb > 0 ? gb : 1;
    const int g = d / (dim / n_groups);
    const size_t row = ((size_t)b * dim + d) * (size_t)seqlen;
    REAL h[256];
    for (int n = 0; n < dstate; ++n) h[n] = 0;
    const REAL dval = Dv ? (REAL)Dv[d] : 0;
    const REAL bval = bias ? (REAL)bias[d] : 0;
    for (int t = 0; t < seqlen; ++t) {
        const REAL ut = (REAL)u[row + t];
        REAL dt = (REAL)delta[row + t] + bval;
        if (softplus) dt = dt <= (REAL)20 ? LOG1P(EXP(dt)) : dt;
        const REAL du = dt * ut;
        REAL y = dval * ut;
        for (int n = 0; n < dstate; ++n) {
            const REAL a = EXP(dt * (REAL)A[(size_t)d * dstate + n]);
            REAL bterm, cterm;
            if (gb > 0) {
                bterm = (REAL)Bm[(((size_t)b * gb + g) * dstate + n) * seqlen + t] * du;
            } else {
                bterm = du;
            }
            if (gc > 0) {
                const REAL cv = (REAL)Cm[(((size_t)b * gc + g) * dstate + n) * seqlen + t];
                cterm = gb > 0 ? cv : (REAL)Bm[(size_t)d * dstate + n] * cv;
            } else {
                const REAL cc = (REAL)Cm[(size_t)d * dstate + n];
                cterm = gb > 0 ? cc : (REAL)Bm[(size_t)d * dstate + n] * cc;
            }
            h[n] = a * h[n] + bterm;
            y += h[n] * cterm;
        }
        if (gate) {
            const REAL zt = (REAL)z[row + t];
            y *= zt / ((REAL)1 + EXP(-zt));
        }
        out[row + t] = (OUT_T)y;
    }
    /* the state after the last token (the extension output return_last_state) */
    if (last)
        for (int n = 0; n < dstate; ++n) last[((size_t)b * dim + d) * (size_t)dstate + n] = (OUT_T)h[n];
}

int FN(oracle_ss)(int batch, int dim, int seqlen, int dstate, int gb, int gc, const float *u,
                  const float *delta, const float *A, const float *Bm, const float *Cm, const float *Dv,
                  const float *z, const float *bias, int softplus, int gate, OUT_T *out, OUT_T *last,
                  int nthreads) {
    if (batch <= 0 || dim <= 0 || seqlen <= 0 || dstate <= 0 || dstate > 256) return 1;
    const int n_groups = gb > 0 ? gb : 1;
    if (dim % n_groups != 0) return 2;
    if (gate && !z) return 3;
    const long units = (long)batch * dim;
#pragma omp parallel for schedule(dynamic, 4) num_threads(nthreads > 0 ? nthreads : 1)
    for (long i = 0; i < units; ++i) {
        FN(ss_unit)((int)(i / dim), (int)(i % dim), dim, seqlen, dstate, gb, gc, u, delta, A, Bm, Cm, Dv, z, bias,
                    softplus, gate, out, last);
    }
    return 0;
}

/* ------------------------------------------------------------------ GatedDeltaNet2Fn
 * Per (b, h), state S[K][V] = initial_state[b,h] or 0. For each token t
 * (gated_deltanet2_fwd.cu:40-76 preparation, :83-140 recurrence; the generic
 * path :142-233 computes the same):
 *   q^ = q * scale * rsqrt(sum q^2 + 1e-6), k^ = k * rsqrt(sum k^2 + 1e-6) when
 *        use_qk_l2norm_in_kernel, else q^ = q * scale, k^ = k
 *   S[i,:] *= exp(g[t,i])
 *   e_j = sum_i beta[t,i] * k^_i * S[i,j]
 *   u_j = w[t,j] * v[t,j] - e_j
 *   S[i,j] += k^_i * u_j
 *   o[t,j] = sum_i q^_i * S[i,j]
 */
static void FN(gdn_unit)(int b, int h, int T, int H, int K, int V, const float *q, const float *k,
                         const float *v, const float *g, const float *beta, const float *w, const float *init,
                         float scale, int l2norm, OUT_T *out, OUT_T *final_state, REAL *S, REAL *qh,
                         REAL *kh) {
    const size_t state_base = ((size_t)b * H + h) * (size_t)K * V;
    for (size_t i = 0; i < (size_t)K * V; ++i) S[i] = init ? (REAL)init[state_base + i] : 0;
    for (int t = 0; t < T; ++t) {
        const size_t qk_base = (((size_t)b * T + t) * H + h) * (size_t)K;
        const size_t vv_base = (((size_t)b * T + t) * H + h) * (size_t)V;
        REAL qn = 0, kn = 0;
        for (int i = 0; i < K; ++i) {
            qn += (REAL)q[qk_base + i] * (REAL)q[qk_base + i];
            kn += (REAL)k[qk_base + i] * (REAL)k[qk_base + i];
        }
        REAL qmul = (REAL)scale, kmul = 1;
        if (l2norm) {
            qmul *= (REAL)1 / SQRT(qn + (REAL)1e-6);
            kmul = (REAL)1 / SQRT(kn + (REAL)1e-6);
        }
        for (int i = 0; i < K; ++i) {
            qh[i] = (REAL)q[qk_base + i] * qmul;
            kh[i] = (REAL)k[qk_base + i] * kmul;
        }
        for (int i = 0; i < K; ++i) {
            const REAL dec = EXP((REAL)g[qk_base + i]);
            REAL *row = S + (size_t)i * V;
            for (int j = 0; j < V; ++j) row[j] *= dec;
        }
        for (int j = 0; j < V; ++j) {
            REAL e = 0;
            for (int i = 0; i < K; ++i) e += (REAL)beta[qk_base + i] * kh[i] * S[(size_t)i * V + j];
            const REAL uj = (REAL)w[vv_base + j] * (REAL)v[vv_base + j] - e;
            for (int i = 0; i < K; ++i) S[(size_t)i * V + j] += kh[i] * uj;
        }
        for (int j = 0; j < V; ++j) {
            REAL o = 0;
            for (int i = 0; i < K; ++i) o += qh[i] * S[(size_t)i * V + j];
            out[vv_base + j] = (OUT_T)o;
        }
    }
    /* the state after the last token (the extension output output_final_state) */
    if (final_state)
        for (size_t i = 0; i < (size_t)K * V; ++i) final_state[state_base + i] = (OUT_T)S[i];
}

int FN(oracle_gdn)(int B, int T, int H, int K, int V, const float *q, const float *k, const float *v,
                   const float *g, const float *beta, const float *w, const float *init, float scale, int l2norm,
                   OUT_T *out, OUT_T *final_state, int nthreads) {
    if (B <= 0 || T <= 0 || H <= 0 || K <= 0 || V <= 0) return 1;
    const long units = (long)B * H;
    int rc = 0;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
    {
        REAL *S = (REAL *)malloc(sizeof(REAL) * (size_t)K * V);
        REAL *qh = (REAL *)malloc(sizeof(REAL) * (size_t)K);
        REAL *kh = (REAL *)malloc(sizeof(REAL) * (size_t)K);
        if (!S || !qh || !kh) {
#pragma omp atomic write
            rc = 4;
        } else {
#pragma omp for schedule(dynamic, 1)
            for (long i = 0; i < units; ++i) {
                FN(gdn_unit)((int)(i / H), (int)(i % H), T, H, K, V, q, k, v, g, beta, w, init, scale, l2norm, out,
                             final_state, S, qh, kh);
            }
        }
        free(S);
        free(qh);
        free(kh);
    }
    return rc;
}

/* ------------------------------------------------------------------ Mamba3SisoFn
 * Per (b, h) with g = h / (H / G): S[P][N] = 0, theta[A] = 0. For each token t
 * (mamba3_siso_fwd.cu:50-172):
 *   theta_a = wrap(theta_a + tanh(Angles[b,t,h,a]) * DT[b,h,t] * pi),
 *             wrap(x) = x - 2pi * floor(x / 2pi)                     (:82-86, :26-28)
 *   q = Q[b,t,g,:] + Q_bias[h,:], k = K[b,t,g,:] + K_bias[h,:], qk = q . k  (:89-106)
 *   rotate pairs (2p, 2p+1) by theta_p for p < A, by 0 otherwise           (:108-124)
 *   gamma = DT_t * sigmoid(Trap_t); gamma' = DT_{t+1} * (1 - sigmoid(Trap_{t+1}))
 *           for t + 1 < T, else 0; scale = gamma + gamma'                  (:126-138)
 *   S *= exp(ADT_t)                                                       (:140-143)
 *   o_p = sum_i q_rot_i S[p,i] + (D_h + qk * gamma) * V_p, times silu(Z_p)  (:146-161)
 *   S[p,i] += V_p * k_rot_i * scale                                       (:164-169)
 */
/* Recurrent states (the extension inputs / outputs has_input_states and
 * return_final_states; the reference rejects both): per (b, h) the state
 * S [P][N], the wrapped angles theta [A], and the last token's rotated k [N]
 * and v [P]. The trapezoid term looks one token ahead, so the last token of a
 * call adds v k^T gamma only (gamma' = 0 there); a continuation adds the
 * missing v_prev k_prev^T DT_0 (1 - sigmoid(Trap_0)) before its first token,
 * which makes two chained calls equal one call over both parts. */
typedef struct {
    const float *s, *angle, *k, *v; /* input states (null: zero start) */
    OUT_T *s_out, *angle_out, *k_out, *v_out; /* final states (null: not requested) */
} FN(m3_states);

static void FN(m3_unit)(int b, int h, int T, int H, int G, int N, int P, int A, const float *Q, const float *Kt,
                        const float *Vt, const float *ADT, const float *DT, const float *Trap, const float *Qb,
                        const float *Kb, const float *Ang, const float *Dv, const float *Z, OUT_T *out, REAL *S,
                        REAL *theta, REAL *qr, REAL *kr, const FN(m3_states) *st) {
    const REAL pi = (REAL)3.14159265358979323846;
    const REAL two_pi = (REAL)2 * pi;
    const int g = h / (H / G);
    const size_t hb = (size_t)b * H + h;
    const size_t bh = hb * (size_t)T;
    for (size_t i = 0; i < (size_t)P * N; ++i) S[i] = st && st->s ? (REAL)st->s[hb * P * N + i] : 0;
    for (int a = 0; a < A; ++a) theta[a] = st && st->angle ? (REAL)st->angle[hb * A + a] : 0;
    if (st && st->s && T > 0) {
        const REAL gprev = (REAL)DT[bh] * ((REAL)1 - (REAL)1 / ((REAL)1 + EXP(-(REAL)Trap[bh])));
        for (int p = 0; p < P; ++p)
            for (int i = 0; i < N; ++i)
                S[(size_t)p * N + i] += (REAL)st->v[hb * P + p] * (REAL)st->k[hb * N + i] * gprev;
    }
    for (int t = 0; t < T; ++t) {
        const REAL dt = (REAL)DT[bh + t];
        for (int a = 0; a < A; ++a) {
            const REAL raw = (REAL)Ang[(((size_t)b * T + t) * H + h) * (size_t)A + a];
            const REAL nx = theta[a] + TANH(raw) * dt * pi;
            theta[a] = nx - two_pi * FLOOR(nx / two_pi);
        }
        const size_t qb = (((size_t)b * T + t) * G + g) * (size_t)N;
        REAL qk = 0;
        for (int i = 0; i < N; ++i) {
            qr[i] = (REAL)Q[qb + i] + (REAL)Qb[(size_t)h * N + i];
            kr[i] = (REAL)Kt[qb + i] + (REAL)Kb[(size_t)h * N + i];
            qk += qr[i] * kr[i];
        }
        for (int p = 0; p < N / 2; ++p) {
            const REAL th = p < A ? theta[p] : 0;
            const REAL c = COS(th), s = SIN(th);
            const REAL q0 = qr[2 * p], q1 = qr[2 * p + 1], k0 = kr[2 * p], k1 = kr[2 * p + 1];
            qr[2 * p] = q0 * c - q1 * s;
            qr[2 * p + 1] = q0 * s + q1 * c;
            kr[2 * p] = k0 * c - k1 * s;
            kr[2 * p + 1] = k0 * s + k1 * c;
        }
        const REAL gamma = dt * ((REAL)1 / ((REAL)1 + EXP(-(REAL)Trap[bh + t])));
        REAL gshift = 0;
        if (t + 1 < T) {
            gshift = (REAL)DT[bh + t + 1] * ((REAL)1 - (REAL)1 / ((REAL)1 + EXP(-(REAL)Trap[bh + t + 1])));
        }
        const REAL scl = gamma + gshift;
        const REAL decay = EXP((REAL)ADT[bh + t]);
        for (size_t i = 0; i < (size_t)P * N; ++i) S[i] *= decay;
        const REAL diag = (Dv ? (REAL)Dv[h] : 0) + qk * gamma;
        const size_t vb = (((size_t)b * T + t) * H + h) * (size_t)P;
        for (int p = 0; p < P; ++p) {
            REAL acc = 0;
            const REAL *srow = S + (size_t)p * N;
            for (int i = 0; i < N; ++i) acc += qr[i] * srow[i];
            REAL o = acc + diag * (REAL)Vt[vb + p];
            if (Z) {
                const REAL zv = (REAL)Z[vb + p];
                o *= zv / ((REAL)1 + EXP(-zv));
            }
            out[vb + p] = (OUT_T)o;
        }
        for (int p = 0; p < P; ++p) {
            const REAL vp = (REAL)Vt[vb + p];
            REAL *srow = S + (size_t)p * N;
            for (int i = 0; i < N; ++i) srow[i] += vp * (kr[i] * scl);
        }
        if (t == T - 1 && st) {
            if (st->k_out)
                for (int i = 0; i < N; ++i) st->k_out[hb * N + i] = (OUT_T)kr[i];
            if (st->v_out)
                for (int p = 0; p < P; ++p) st->v_out[hb * P + p] = (OUT_T)Vt[vb + p];
        }
    }
    if (st && st->s_out)
        for (size_t i = 0; i < (size_t)P * N; ++i) st->s_out[hb * P * N + i] = (OUT_T)S[i];
    if (st && st->angle_out)
        for (int a = 0; a < A; ++a) st->angle_out[hb * A + a] = (OUT_T)theta[a];
}

int FN(oracle_m3)(int B, int T, int H, int G, int N, int P, int A, const float *Q, const float *K, const float *V,
                  const float *ADT, const float *DT, const float *Trap, const float *Qb, const float *Kb,
                  const float *Ang, const float *Dv, const float *Z, OUT_T *out, const float *s_in,
                  const float *angle_in, const float *k_in, const float *v_in, OUT_T *s_out, OUT_T *angle_out,
                  OUT_T *k_out, OUT_T *v_out, int nthreads) {
    FN(m3_states) st = {s_in, angle_in, k_in, v_in, s_out, angle_out, k_out, v_out};
    if (B <= 0 || T <= 0 || H <= 0 || G <= 0 || N <= 0 || P <= 0 || A <= 0) return 1;
    if (H % G != 0 || N % 2 != 0 || A > N / 2) return 2;
    const long units = (long)B * H;
    int rc = 0;
#pragma omp parallel num_threads(nthreads > 0 ? nthreads : 1)
    {
        REAL *S = (REAL *)malloc(sizeof(REAL) * (size_t)P * N);
        REAL *theta = (REAL *)malloc(sizeof(REAL) * (size_t)A);
        REAL *qr = (REAL *)malloc(sizeof(REAL) * (size_t)N);
        REAL *kr = (REAL *)malloc(sizeof(REAL) * (size_t)N);
        if (!S || !theta || !qr || !kr) {
#pragma omp atomic write
            rc = 4;
        } else {
#pragma omp for schedule(dynamic, 1)
            for (long i = 0; i < units; ++i) {
                FN(m3_unit)((int)(i / H), (int)(i % H), T, H, G, N, P, A, Q, K, V, ADT, DT, Trap, Qb, Kb, Ang, Dv, Z,
                            out, S, theta, qr, kr, &st);
            }
        }
        free(S);
        free(theta);
        free(qr);
        free(kr);
    }
    return rc;
}
