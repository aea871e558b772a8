/* k3_oracle.c -- CPU restatement of the kimi-k3-in-c attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see k3_oracle.h). Written from the reference's documented
 * algorithm; each function names the reference lines it restates. Build with
 * -ffp-contract=off like the reference (Makefile:136-140 of the reference), so that the
 * fp32 recurrence rounds exactly as k3_kda_step does.
 */
#include "k3_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static inline float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

/* ------------------------------------------------------------------------------------
 * k3_kda_step (src/core/k3_ops.c:186-243). Same four passes in the same order so the
 * fp32 rounding matches: decay rows, u = S^T k, rank-one delta write, o = S^T q from the
 * updated state. Zero k_i / q_i rows are skipped exactly as the reference skips them. */
void orc_kda_step(float *S, float *o, const float *q, const float *k, const float *v,
                  const float *alpha, float beta, int dk, int dv)
{
    float ustack[512];
    float *u = dv <= 512 ? ustack : (float *)calloc((size_t)dv, sizeof(float));
    if (!u) abort();
    for (int i = 0; i < dk; i++) {
        float *row = S + (size_t)i * dv;
        const float a = alpha[i];
        for (int j = 0; j < dv; j++) row[j] *= a;
    }
    for (int j = 0; j < dv; j++) u[j] = 0.0f;
    for (int i = 0; i < dk; i++) {
        const float ki = k[i];
        if (ki == 0.0f) continue;
        const float *row = S + (size_t)i * dv;
        for (int j = 0; j < dv; j++) u[j] += ki * row[j];
    }
    for (int i = 0; i < dk; i++) {
        const float ki = k[i];
        if (ki == 0.0f) continue;
        float *row = S + (size_t)i * dv;
        for (int j = 0; j < dv; j++) row[j] += ki * beta * (v[j] - u[j]);
    }
    for (int j = 0; j < dv; j++) o[j] = 0.0f;
    for (int i = 0; i < dk; i++) {
        const float qi = q[i];
        if (qi == 0.0f) continue;
        const float *row = S + (size_t)i * dv;
        for (int j = 0; j < dv; j++) o[j] += qi * row[j];
    }
    if (u != ustack) free(u);
}

/* ------------------------------------------------------------------------------------
 * Recurrence driver of k3_kda_layer (src/core/k3_ops.c:908-938): per head, t in order,
 * q scaled by q_scale into a private row, alpha per (t, h, channel), beta per (t, h).
 * Sequences of a packed batch are independent streams with their own state. */
void orc_kda_recurrence(float *S, float *o, const float *q, const float *k,
                        const float *v, const float *gate, int gate_is_log,
                        const float *beta, const int *cu_seqlens, int nseq, int H,
                        int dk, int dv, float q_scale, int nthreads)
{
    const long nstream = (long)nseq * H;
#ifdef _OPENMP
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
#endif
    for (long sh = 0; sh < nstream; sh++) {
        const int n = (int)(sh / H), h = (int)(sh % H);
        float *St;
        float *own = NULL;
        if (S) {
            St = S + ((size_t)n * H + h) * (size_t)dk * dv;
        } else {
            own = (float *)calloc((size_t)dk * dv, sizeof(float));
            if (!own) abort();
            St = own;
        }
        float *qs = (float *)malloc((size_t)dk * sizeof(float));
        float *al = (float *)malloc((size_t)dk * sizeof(float));
        if (!qs || !al) abort();
        for (int t = cu_seqlens[n]; t < cu_seqlens[n + 1]; t++) {
            const size_t offk = ((size_t)t * H + h) * dk;
            const size_t offv = ((size_t)t * H + h) * dv;
            for (int i = 0; i < dk; i++) qs[i] = q[offk + i] * q_scale;
            for (int i = 0; i < dk; i++)
                al[i] = gate_is_log ? expf(gate[offk + i]) : gate[offk + i];
            orc_kda_step(St, o + offv, qs, k + offk, v + offv, al,
                         beta[(size_t)t * H + h], dk, dv);
        }
        free(qs); free(al); free(own);
    }
}

/* k3_kda_decay (src/core/k3_ops.c:167-183): A_log per head. */
void orc_kda_decay(float *g, float *alpha, const float *z, const float *A_log,
                   const float *dt_bias, int H, int D, float lb)
{
    for (int h = 0; h < H; h++) {
        const float a = expf(A_log[h]);
        for (int d = 0; d < D; d++) {
            const int i = h * D + d;
            const float gi = lb * sigm(a * (z[i] + dt_bias[i]));
            g[i] = gi;
            alpha[i] = expf(gi);
        }
    }
}

/* k3_rmsnorm (src/core/k3_ops.c:94-101). */
void orc_rmsnorm(float *y, const float *x, const float *w, int n, float eps)
{
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)x[i] * (double)x[i];
    const float inv = (float)(1.0 / sqrt(ss / (double)n + (double)eps));
    for (int i = 0; i < n; i++) y[i] = w[i] * x[i] * inv;
}

/* l2norm_ (src/core/k3_ops.c:845-851). */
void orc_l2norm(float *v, int n, float eps)
{
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double)v[i] * (double)v[i];
    const float inv = (float)(1.0 / sqrt(ss + (double)eps));
    for (int i = 0; i < n; i++) v[i] *= inv;
}

/* k3_shortconv (src/core/k3_ops.c:133-165): taps oldest..newest, w[k-1] multiplies the
 * current input, history shifted left, SiLU fused. */
void orc_shortconv(float *y, const float *x, const float *w, float *state,
                   int channels, int k, int T)
{
    const int hist = k - 1;
    float buf[64];
    if (hist > 64) abort();
    for (int c = 0; c < channels; c++) {
        for (int j = 0; j < hist; j++) buf[j] = state ? state[(size_t)c * hist + j] : 0.0f;
        for (int t = 0; t < T; t++) {
            const float cur = x[(size_t)t * channels + c];
            float acc = w[(size_t)c * k + hist] * cur;
            for (int j = 0; j < hist; j++) acc += w[(size_t)c * k + j] * buf[j];
            for (int j = 0; j + 1 < hist; j++) buf[j] = buf[j + 1];
            if (hist > 0) buf[hist - 1] = cur;
            y[(size_t)t * channels + c] = acc * sigm(acc);
        }
        if (state)
            for (int j = 0; j < hist; j++) state[(size_t)c * hist + j] = buf[j];
    }
}

/* y[out] = W[out][in] . x, double accumulator (the reference's k3_matmul accumulates in
 * double too, k3_ops.c:265-291; the partition differs, which is inside fp32 rounding). */
static void mm(float *y, const float *x, const float *W, int in, int out)
{
    for (int r = 0; r < out; r++) {
        const float *row = W + (size_t)r * in;
        double acc = 0.0;
        for (int i = 0; i < in; i++) acc += (double)row[i] * (double)x[i];
        y[r] = (float)acc;
    }
}

/* k3_kda_layer (src/core/k3_ops.c:864-951), fp32 weights, steps 1-9 in the same order. */
void orc_kda_layer(float *out, const float *x, int T, int E, int H, int D,
                   int K, float lb, float eps,
                   const float *Wq, const float *Wk, const float *Wv,
                   const float *q_conv, const float *k_conv, const float *v_conv,
                   const float *f_a, const float *f_b, const float *A_log,
                   const float *dt_bias, const float *Wb, const float *Wg,
                   const float *o_norm, const float *Wo, float *state)
{
    const int P = H * D, hist = K - 1;
    float *q = (float *)calloc((size_t)T * P, sizeof(float));
    float *k = (float *)calloc((size_t)T * P, sizeof(float));
    float *v = (float *)calloc((size_t)T * P, sizeof(float));
    float *z = (float *)calloc((size_t)T * P, sizeof(float));
    float *al = (float *)calloc((size_t)T * P, sizeof(float));
    float *bt = (float *)calloc((size_t)T * H, sizeof(float));
    float *o = (float *)calloc((size_t)T * P, sizeof(float));
    float *gb = (float *)calloc((size_t)P, sizeof(float));
    float *fa = (float *)calloc((size_t)D, sizeof(float));
    if (!q || !k || !v || !z || !al || !bt || !o || !gb || !fa) abort();

    /* 1. projections (k3_ops.c:877-886) */
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * E;
        mm(q + (size_t)t * P, xt, Wq, E, P);
        mm(k + (size_t)t * P, xt, Wk, E, P);
        mm(v + (size_t)t * P, xt, Wv, E, P);
        mm(bt + (size_t)t * H, xt, Wb, E, H);
        mm(fa, xt, f_a, E, D);
        mm(z + (size_t)t * P, fa, f_b, D, P);
    }
    /* 2. ShortConv, state after the recurrent block (k3_ops.c:889-892) */
    float *cs = state ? state + (size_t)H * D * D : NULL;
    orc_shortconv(q, q, q_conv, cs, P, K, T);
    orc_shortconv(k, k, k_conv, cs ? cs + (size_t)P * hist : NULL, P, K, T);
    orc_shortconv(v, v, v_conv, cs ? cs + (size_t)2 * P * hist : NULL, P, K, T);
    /* 3. L2 on q and k only (k3_ops.c:895-899) */
    for (int t = 0; t < T; t++)
        for (int h = 0; h < H; h++) {
            orc_l2norm(q + (size_t)t * P + (size_t)h * D, D, 1e-6f);
            orc_l2norm(k + (size_t)t * P + (size_t)h * D, D, 1e-6f);
        }
    /* 4/5. beta, decay (k3_ops.c:902-906) */
    for (int t = 0; t < T; t++) {
        for (int h = 0; h < H; h++) bt[(size_t)t * H + h] = sigm(bt[(size_t)t * H + h]);
        orc_kda_decay(z + (size_t)t * P, al + (size_t)t * P, z + (size_t)t * P, A_log,
                      dt_bias, H, D, lb);
    }
    /* 6. recurrence (k3_ops.c:908-938) */
    int cu[2] = {0, T};
    orc_kda_recurrence(state, o, q, k, v, al, 0, bt, cu, 1, H, D, D,
                       1.0f / sqrtf((float)D), 1);
    /* 7/8/9. head RMSNorm, then gate, then o_proj (k3_ops.c:941-949) */
    for (int t = 0; t < T; t++) {
        const float *xt = x + (size_t)t * E;
        float *ot = o + (size_t)t * P;
        for (int h = 0; h < H; h++)
            orc_rmsnorm(ot + (size_t)h * D, ot + (size_t)h * D, o_norm, D, eps);
        mm(gb, xt, Wg, E, P);
        for (int i = 0; i < P; i++) ot[i] *= sigm(gb[i]);
        mm(out + (size_t)t * E, ot, Wo, P, E);
    }
    free(q); free(k); free(v); free(z); free(al); free(bt); free(o); free(gb); free(fa);
}

/* ------------------------------------------------------------------------------------
 * Absorbed MLA decode. The reference loop (src/core/k3_ops.c:381-411) per head:
 *   score[s] = (float)(sum_i q_nope_i k_s,i + sum_i q_rope_i kr_s,i in double) * scale
 *   m = max score; p_s = expf(score - m); z = sum p_s in double
 *   o = sum_s (float)(p_s / z) * v_s
 * with k_s = W_UK c_s and v_s = W_UV c_s. Absorbed: q_nope . (W_UK c_s) =
 * (W_UK^T q_nope) . c_s and sum_s p_s (W_UV c_s) = W_UV (sum_s p_s c_s). Both absorbed
 * products and the latent accumulation run in double here, which is at least as
 * accurate as the reference's expanded fp32 cache. */
void orc_mla_absorbed_decode(float *out, const float *q_nope, const float *q_rope,
                             const float *latent, const float *rope,
                             const float *w_uk, const float *w_uv,
                             const int *ctx_lens, int B, int cap, int H, int dn,
                             int dr, int dl, int dv, float scale, int nthreads)
{
    const long nwork = (long)B * H;
#ifdef _OPENMP
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nthreads)
#endif
    for (long bh = 0; bh < nwork; bh++) {
        const int b = (int)(bh / H), h = (int)(bh % H);
        const int P = ctx_lens[b];
        const float *qn = q_nope + ((size_t)b * H + h) * dn;
        const float *qr = q_rope + ((size_t)b * H + h) * dr;
        const float *Wk = w_uk + (size_t)h * dn * dl;
        const float *Wv = w_uv + (size_t)h * dv * dl;
        double *qlat = (double *)calloc((size_t)dl, sizeof(double));
        double *olat = (double *)calloc((size_t)dl, sizeof(double));
        float *sc = (float *)malloc((size_t)(P > 0 ? P : 1) * sizeof(float));
        if (!qlat || !olat || !sc) abort();
        for (int i = 0; i < dn; i++) {
            const double qi = qn[i];
            const float *row = Wk + (size_t)i * dl;
            for (int l = 0; l < dl; l++) qlat[l] += qi * (double)row[l];
        }
        float m = -INFINITY;
        for (int s = 0; s < P; s++) {
            const float *c = latent + ((size_t)b * cap + s) * dl;
            const float *kr = rope + ((size_t)b * cap + s) * dr;
            double d = 0.0;
            for (int l = 0; l < dl; l++) d += qlat[l] * (double)c[l];
            for (int i = 0; i < dr; i++) d += (double)qr[i] * (double)kr[i];
            sc[s] = (float)d * scale;
            if (sc[s] > m) m = sc[s];
        }
        double z = 0.0;
        for (int s = 0; s < P; s++) { sc[s] = expf(sc[s] - m); z += sc[s]; }
        for (int s = 0; s < P; s++) {
            const double p = (double)(float)(sc[s] / z);
            const float *c = latent + ((size_t)b * cap + s) * dl;
            for (int l = 0; l < dl; l++) olat[l] += p * (double)c[l];
        }
        float *o = out + ((size_t)b * H + h) * dv;
        for (int j = 0; j < dv; j++) {
            const float *row = Wv + (size_t)j * dl;
            double acc = 0.0;
            for (int l = 0; l < dl; l++) acc += (double)row[l] * olat[l];
            o[j] = (float)acc;
        }
        free(qlat); free(olat); free(sc);
    }
}

/* ------------------------------------------------------------------------------------
 * Chunkwise restatement in double. Within a chunk of C tokens with cumulative log decay
 * G_t = sum_{u<=t} g_u (per key channel), the delta rule unrolls to
 *   (I + Akk) Delta = diag(beta) (V - Ktilde S0),   Ktilde_t = exp(G_t) . k_t
 *   O = Qtilde S0 + Aqk Delta,                      Qtilde_t = exp(G_t) . q_t
 *   S_C = diag(exp(G_C)) S0 + Kbar^T Delta,         Kbar_s = exp(G_C - G_s) . k_s
 * with Akk[t][s] = beta_t sum_i k_t,i k_s,i exp(G_t,i - G_s,i) for s < t and
 * Aqk[t][s] = sum_i q_t,i k_s,i exp(G_t,i - G_s,i) for s <= t. Delta is solved by
 * forward substitution (the unit-lower-triangular inverse). */
void orc_kda_chunked_f64(float *o, float *S, double *Akk, double *Aqk,
                         const float *q, const float *k, const float *v,
                         const float *g, const float *beta, int T, int C, int dk,
                         int dv, float q_scale)
{
    double *S0 = (double *)calloc((size_t)dk * dv, sizeof(double));
    double *G = (double *)malloc((size_t)C * dk * sizeof(double));
    double *R = (double *)malloc((size_t)C * dv * sizeof(double));
    double *Dl = (double *)malloc((size_t)C * dv * sizeof(double));
    if (!S0 || !G || !R || !Dl) abort();
    const int nchunk = T / C;
    for (int n = 0; n < nchunk; n++) {
        const int t0 = n * C;
        double *akk = Akk + (size_t)n * C * C, *aqk = Aqk + (size_t)n * C * C;
        for (int i = 0; i < dk; i++) {
            double acc = 0.0;
            for (int t = 0; t < C; t++) {
                acc += (double)g[(size_t)(t0 + t) * dk + i];
                G[(size_t)t * dk + i] = acc;
            }
        }
        for (int t = 0; t < C; t++)
            for (int s = 0; s < C; s++) {
                double a = 0.0, b = 0.0;
                if (s <= t)
                    for (int i = 0; i < dk; i++) {
                        const double e = exp(G[(size_t)t * dk + i] - G[(size_t)s * dk + i]);
                        const double ks = k[(size_t)(t0 + s) * dk + i];
                        a += (double)k[(size_t)(t0 + t) * dk + i] * ks * e;
                        b += (double)q[(size_t)(t0 + t) * dk + i] * q_scale * ks * e;
                    }
                akk[(size_t)t * C + s] = s < t ? (double)beta[t0 + t] * a : 0.0;
                aqk[(size_t)t * C + s] = s <= t ? b : 0.0;
            }
        /* R = diag(beta) (V - Ktilde S0) */
        for (int t = 0; t < C; t++)
            for (int j = 0; j < dv; j++) {
                double ks0 = 0.0;
                for (int i = 0; i < dk; i++)
                    ks0 += exp(G[(size_t)t * dk + i]) * (double)k[(size_t)(t0 + t) * dk + i] *
                           S0[(size_t)i * dv + j];
                R[(size_t)t * dv + j] =
                    (double)beta[t0 + t] * ((double)v[(size_t)(t0 + t) * dv + j] - ks0);
            }
        /* forward substitution: Delta_t = R_t - sum_{s<t} Akk[t][s] Delta_s */
        for (int t = 0; t < C; t++)
            for (int j = 0; j < dv; j++) {
                double d = R[(size_t)t * dv + j];
                for (int s = 0; s < t; s++) d -= akk[(size_t)t * C + s] * Dl[(size_t)s * dv + j];
                Dl[(size_t)t * dv + j] = d;
            }
        /* outputs */
        for (int t = 0; t < C; t++)
            for (int j = 0; j < dv; j++) {
                double acc = 0.0;
                for (int i = 0; i < dk; i++)
                    acc += exp(G[(size_t)t * dk + i]) * (double)q[(size_t)(t0 + t) * dk + i] *
                           q_scale * S0[(size_t)i * dv + j];
                for (int s = 0; s <= t; s++) acc += aqk[(size_t)t * C + s] * Dl[(size_t)s * dv + j];
                o[(size_t)(t0 + t) * dv + j] = (float)acc;
            }
        /* state to the chunk end */
        for (int i = 0; i < dk; i++) {
            const double gC = G[(size_t)(C - 1) * dk + i];
            for (int j = 0; j < dv; j++) {
                double acc = exp(gC) * S0[(size_t)i * dv + j];
                for (int s = 0; s < C; s++)
                    acc += exp(gC - G[(size_t)s * dk + i]) *
                           (double)k[(size_t)(t0 + s) * dk + i] * Dl[(size_t)s * dv + j];
                S0[(size_t)i * dv + j] = acc;
            }
        }
    }
    for (size_t i = 0; i < (size_t)dk * dv; i++) S[i] = (float)S0[i];
    free(S0); free(G); free(R); free(Dl);
}

/* ------------------------------------------------------------------------------------
 * MXFP4. E2M1 is 1 sign, 2 exponent, 1 mantissa bits: magnitudes 0, .5, 1, 1.5, 2, 3, 4, 6
 * by the low three bits, bit 3 the sign (code 8 is -0). E8M0 is a bare biased exponent. */
static float e2m1(unsigned nib)
{
    static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
    const float m = mag[nib & 7u];
    return (nib & 8u) ? -m : m;
}

static float e8m0(unsigned char s) { return s == 255 ? 0.0f : ldexpf(1.0f, (int)s - 127); }

void orc_mxfp4_dequant(float *out, const unsigned char *packed, const unsigned char *scales,
                       int rows, int in, int group)
{
    const int ngrp = (in + group - 1) / group;
    for (int r = 0; r < rows; r++)
        for (int i = 0; i < in; i++) {
            const unsigned char byte = packed[(size_t)r * (in / 2) + i / 2];
            const unsigned nib = (i & 1) ? (unsigned)(byte >> 4) : (unsigned)(byte & 15);
            out[(size_t)r * in + i] = e2m1(nib) * e8m0(scales[(size_t)r * ngrp + i / group]);
        }
}

void orc_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                      const unsigned char *scales, int in, int rows, int T, int group)
{
    const int ngrp = (in + group - 1) / group;
    for (int t = 0; t < T; t++)
        for (int r = 0; r < rows; r++) {
            double acc = 0.0;
            for (int i = 0; i < in; i++) {
                const unsigned char byte = packed[(size_t)r * (in / 2) + i / 2];
                const unsigned nib = (i & 1) ? (unsigned)(byte >> 4) : (unsigned)(byte & 15);
                const double w = (double)e2m1(nib) *
                                 (double)e8m0(scales[(size_t)r * ngrp + i / group]);
                acc += w * (double)x[(size_t)t * in + i];
            }
            y[(size_t)t * rows + r] = (float)acc;
        }
}
