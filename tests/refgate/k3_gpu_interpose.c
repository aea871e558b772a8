/* k3_gpu_interpose.c -- routes the reference's hot-path calls to the B200 drop-ins.
 *
 * This is the one-line switch INTEGRATION.md describes, made without editing a reference
 * source: the reference's src/core/k3_ops.c is built unmodified as a shared library, and
 * this library, linked ahead of it, defines the same three global functions. The dynamic
 * linker binds every call -- the test's own and the ones inside k3_ops.c, which go through
 * the PLT because the library is position-independent with default visibility -- to the
 * first definition, this one:
 *
 *   k3_kda_step   (include/k3/k3.h:164-165)  -> k3g_kda_step
 *   k3_kda_layer  (include/k3/k3.h:468-469)  -> k3g_kda_layer
 *   k3_mla_cached (include/k3/k3.h:219-221)  -> k3g_mla_cached
 *
 * so k3_decoder_layer_inc (k3_ops.c:1030-1031) and k3_mla (:426-430) reach the GPU too. The
 * casts are exact because k3_gpu.h's structs are K3Cfg / K3KdaW / K3MlaW field for field;
 * the static assertions below check that against the reference's own header at build time.
 * At exit it prints how many calls it routed, so a gate run proves the GPU path ran.
 *
 * Test infrastructure: built by tests/refgate/Makefile from the reference checkout, never
 * part of libk3cuda or libk3gpu.
 */
#include <stddef.h>
#include <stdio.h>
#include <stdlib.h>

#include "k3.h"
#include "k3_gpu.h"

#define SAME(T1, T2, f) _Static_assert(offsetof(T1, f) == offsetof(T2, f), #T1 "." #f)
_Static_assert(sizeof(K3Cfg) == sizeof(k3g_cfg), "K3Cfg size");
SAME(K3Cfg, k3g_cfg, hidden); SAME(K3Cfg, k3g_cfg, rms_eps); SAME(K3Cfg, k3g_cfg, kda_heads);
SAME(K3Cfg, k3g_cfg, kda_head_dim); SAME(K3Cfg, k3g_cfg, conv_k); SAME(K3Cfg, k3g_cfg, gate_lb);
SAME(K3Cfg, k3g_cfg, n_heads); SAME(K3Cfg, k3g_cfg, q_lora); SAME(K3Cfg, k3g_cfg, kv_lora);
SAME(K3Cfg, k3g_cfg, qk_nope); SAME(K3Cfg, k3g_cfg, qk_rope); SAME(K3Cfg, k3g_cfg, v_head);
SAME(K3Cfg, k3g_cfg, situ_b2); SAME(K3Cfg, k3g_cfg, full_attn);
_Static_assert(sizeof(K3KdaW) == sizeof(k3g_kda_weights), "K3KdaW size");
SAME(K3KdaW, k3g_kda_weights, q); SAME(K3KdaW, k3g_kda_weights, f_a);
SAME(K3KdaW, k3g_kda_weights, A_log); SAME(K3KdaW, k3g_kda_weights, o);
SAME(K3KdaW, k3g_kda_weights, wdt);
_Static_assert(sizeof(K3MlaW) == sizeof(k3g_mla_weights), "K3MlaW size");
SAME(K3MlaW, k3g_mla_weights, kv_b); SAME(K3MlaW, k3g_mla_weights, g);
SAME(K3MlaW, k3g_mla_weights, kv_a_norm); SAME(K3MlaW, k3g_mla_weights, wdt);

static long n_step, n_kda, n_mla;

static void report(void)
{
    fprintf(stderr, "k3gpu-interpose: routed to the GPU: k3_kda_step %ld, k3_kda_layer %ld, "
                    "k3_mla_cached %ld\n", n_step, n_kda, n_mla);
}

static void count(long *n)
{
    if (!n_step && !n_kda && !n_mla) atexit(report);
    (*n)++;
}

void k3_kda_step(float *S, float *o, const float *q, const float *k, const float *v,
                 const float *alpha, float beta, int dk, int dv)
{
    count(&n_step);
    k3g_kda_step(S, o, q, k, v, alpha, beta, dk, dv);
}

void k3_kda_layer(float *out, const float *x, const K3KdaW *w, const K3Cfg *c, int T,
                  float *state, float *scratch)
{
    count(&n_kda);
    k3g_kda_layer(out, x, (const k3g_kda_weights *)w, (const k3g_cfg *)c, T, state, scratch);
}

void k3_mla_cached(float *out, const float *x, const K3MlaW *w, const K3Cfg *c, int T,
                   float *scratch, float *kvc, float *ropec, int cached, int cap)
{
    count(&n_mla);
    k3g_mla_cached(out, x, (const k3g_mla_weights *)w, (const k3g_cfg *)c, T, scratch, kvc,
                   ropec, cached, cap);
}
