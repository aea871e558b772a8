/* ref_driver.c -- loops that drive the UNMODIFIED reference kernels.
 *
 * TEST INFRASTRUCTURE ONLY. Compiled together with the reference's own
 * src/core/k3_ops.c into oracle/_ref/libk3ref.so by oracle/Makefile. It contains no
 * arithmetic of its own: it prepares q * q_scale and alpha = expf(g) exactly as
 * tests/unit/test_ops.c:324-337 and src/core/k3_ops.c:918-938 do, then calls the
 * reference's k3_kda_step once per (stream, token). Streams (sequence x head) run in
 * parallel on OpenMP threads, each in its own serial token order, as k3_kda_layer runs
 * its heads (k3_ops.c:927-938). k3ref_kda_layer fills the configuration and weight
 * structs and calls the reference's k3_kda_layer once.
 */
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif
#include "k3.h"

/* Packed varlen recurrence: q,k [sumT][H][dk], v [sumT][H][dv], gate [sumT][H][dk]
 * (log-decay when gate_is_log, else alpha), beta [sumT][H], S [nseq][H][dk][dv]. */
void k3ref_kda_recurrence(float *S, float *o, const float *q, const float *k,
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
        float *St = S + ((size_t)n * H + h) * (size_t)dk * dv;
        float *qs = (float *)malloc((size_t)dk * sizeof(float));
        float *al = (float *)malloc((size_t)dk * sizeof(float));
        if (!qs || !al) abort();
        for (int t = cu_seqlens[n]; t < cu_seqlens[n + 1]; t++) {
            const size_t offk = ((size_t)t * H + h) * dk;
            const size_t offv = ((size_t)t * H + h) * dv;
            for (int i = 0; i < dk; i++) qs[i] = q[offk + i] * q_scale;
            for (int i = 0; i < dk; i++)
                al[i] = gate_is_log ? expf(gate[offk + i]) : gate[offk + i];
            k3_kda_step(St, o + offv, qs, k + offk, v + offv, al,
                        beta[(size_t)t * H + h], dk, dv);
        }
        free(qs); free(al);
    }
}

/* One decode step over nstream independent (sequence, head) states:
 * q,k [nstream][dk], v [nstream][dv], gate [nstream][dk], beta [nstream],
 * S [nstream][dk][dv], o [nstream][dv]. */
void k3ref_kda_decode(float *S, float *o, const float *q, const float *k,
                      const float *v, const float *gate, int gate_is_log,
                      const float *beta, long nstream, int dk, int dv, float q_scale,
                      int nthreads)
{
#ifdef _OPENMP
    if (nthreads < 1) nthreads = 1;
#pragma omp parallel num_threads(nthreads)
#endif
    {
        float *qs = (float *)malloc((size_t)dk * sizeof(float));
        float *al = (float *)malloc((size_t)dk * sizeof(float));
        if (!qs || !al) abort();
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (long sh = 0; sh < nstream; sh++) {
            for (int i = 0; i < dk; i++) qs[i] = q[(size_t)sh * dk + i] * q_scale;
            for (int i = 0; i < dk; i++)
                al[i] = gate_is_log ? expf(gate[(size_t)sh * dk + i]) : gate[(size_t)sh * dk + i];
            k3_kda_step(S + (size_t)sh * dk * dv, o + (size_t)sh * dv, qs,
                        k + (size_t)sh * dk, v + (size_t)sh * dv, al, beta[sh], dk, dv);
        }
        free(qs); free(al);
    }
}

int k3ref_max_threads(void)
{
#ifdef _OPENMP
    return omp_get_num_procs();
#else
    return 1;
#endif
}

/* One k3_kda_layer call (src/core/k3_ops.c:864-951) on x [T][E]. The config fields it reads
 * (hidden, kda_heads, kda_head_dim, conv_k, gate_lb, rms_eps) are set, the rest zero; the
 * projection weights are fp32 (wdt 0) or bf16 bit patterns (wdt 1); state is the
 * reference's layout (H*D*D recurrent, then 3*H*D*(K-1) conv) or NULL. */
void k3ref_kda_layer(float *out, const float *x, int T, int E, int H, int D, int K,
                     float lb, float eps, const void *Wq, const void *Wk, const void *Wv,
                     const float *q_conv, const float *k_conv, const float *v_conv,
                     const void *f_a, const void *f_b, const float *A_log,
                     const float *dt_bias, const void *Wb, const void *Wg,
                     const float *o_norm, const void *Wo, int wdt, float *state)
{
    K3Cfg c;
    memset(&c, 0, sizeof c);
    c.hidden = E; c.kda_heads = H; c.kda_head_dim = D; c.conv_k = K;
    c.gate_lb = lb; c.rms_eps = eps;
    K3KdaW w;
    memset(&w, 0, sizeof w);
    w.q = Wq; w.k = Wk; w.v = Wv;
    w.q_conv = q_conv; w.k_conv = k_conv; w.v_conv = v_conv;
    w.f_a = f_a; w.f_b = f_b; w.A_log = A_log; w.dt_bias = dt_bias;
    w.b = Wb; w.g = Wg; w.o_norm = o_norm; w.o = Wo; w.wdt = wdt;
    float *scratch = (float *)malloc(k3_kda_scratch(&c, T) * sizeof(float));
    if (!scratch) abort();
    k3_kda_layer(out, x, &w, &c, T, state, scratch);
    free(scratch);
}

/* One k3_mla_cached call (src/core/k3_ops.c:321-424) with the config fields it reads set
 * (hidden, n_heads, qk_nope, qk_rope, v_head, q_lora, kv_lora, rms_eps) and its cached-mode
 * scratch (k3_mla_scratch_cached). kvc [cap][H*(qk_nope+v_head)] and ropec [cap][qk_rope]
 * are the reference's expanded caches; g may be NULL (no gate). */
void k3ref_mla_cached(float *out, const float *x, int T, int E, int H, int q_lora,
                      int kv_lora, int qk_nope, int qk_rope, int v_head, float eps,
                      const void *q_a, const void *q_b, const void *kv_a, const void *kv_b,
                      const void *o, const void *g, const float *q_a_norm,
                      const float *kv_a_norm, int wdt, float *kvc, float *ropec, int cached,
                      int cap)
{
    K3Cfg c;
    memset(&c, 0, sizeof c);
    c.hidden = E; c.n_heads = H; c.qk_nope = qk_nope; c.qk_rope = qk_rope; c.v_head = v_head;
    c.q_lora = q_lora; c.kv_lora = kv_lora; c.rms_eps = eps;
    K3MlaW w;
    memset(&w, 0, sizeof w);
    w.q_a = q_a; w.q_b = q_b; w.kv_a = kv_a; w.kv_b = kv_b; w.o = o; w.g = g;
    w.q_a_norm = q_a_norm; w.kv_a_norm = kv_a_norm; w.wdt = wdt;
    float *scratch = (float *)malloc(k3_mla_scratch_cached(&c, T, cap, 1) * sizeof(float));
    if (!scratch) abort();
    k3_mla_cached(out, x, &w, &c, T, scratch, kvc, ropec, cached, cap);
    free(scratch);
}
