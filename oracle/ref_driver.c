/* ref_driver.c -- loops that drive the UNMODIFIED reference kernels.
 *
 * TEST INFRASTRUCTURE ONLY. Compiled together with the reference's own
 * src/core/k3_ops.c into oracle/_ref/libk3ref.so by oracle/Makefile. It contains no
 * arithmetic of its own: it prepares q * q_scale and alpha = expf(g) exactly as
 * tests/unit/test_ops.c:324-337 and src/core/k3_ops.c:918-938 do, then calls the
 * reference's k3_kda_step once per (stream, token). Streams (sequence x head) run in
 * parallel on OpenMP threads, each in its own serial token order, as k3_kda_layer runs
 * its heads (k3_ops.c:927-938).
 */
#include <math.h>
#include <stdlib.h>
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
