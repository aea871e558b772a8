/* k3_gpu.c -- C99 drop-ins for the reference's hot-path calls (include/k3_gpu.h).
 *
 * Host fp32 buffers in, host fp32 buffers out, exactly as the reference functions take
 * them; the device work is libk3cuda's. One process-wide context and grow-only staging
 * buffers serve every call. Any failure aborts with the library's message, the
 * reference's policy for conditions it cannot recover from (src/core/k3_ops.c:38-78).
 */
#include "k3_gpu.h"

#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "k3cuda.h"
#include "k3_gpu_internal.h"

static k3cuda_ctx *g_ctx = NULL;

typedef struct {
    void *ptr;
    size_t bytes;
} Buf;

enum { B_S, B_O, B_Q, B_K, B_V, B_A, B_B, B_WS, B_LAT, B_ROPE, B_UK, B_UV, B_QN, B_QR, B_N };
static Buf g_buf[B_N];

static void die(const char *what)
{
    fprintf(stderr,
            "k3_gpu: FATAL, %s failed: %s\n"
            "    Aborting rather than returning with the output unwritten.\n",
            what, k3cuda_last_error());
    abort();
}

static void ok(int rc, const char *what)
{
    if (rc != K3CUDA_OK) die(what);
}

static k3cuda_ctx *ctx(void)
{
    if (!g_ctx) {
        const char *dev = getenv("K3CUDA_DEVICE");
        ok(k3cuda_init(dev ? atoi(dev) : 0, &g_ctx), "k3cuda_init");
    }
    return g_ctx;
}

k3cuda_ctx *k3g_ctx(void) { return ctx(); }

static void *dev(int slot, size_t bytes)
{
    Buf *b = &g_buf[slot];
    if (b->bytes < bytes) {
        if (b->ptr) ok(k3cuda_free(ctx(), b->ptr), "k3cuda_free");
        b->ptr = NULL;
        b->bytes = 0;
        ok(k3cuda_malloc(ctx(), &b->ptr, bytes), "k3cuda_malloc");
        b->bytes = bytes;
    }
    return b->ptr;
}

static void *put(int slot, const void *src, size_t bytes)
{
    void *d = dev(slot, bytes);
    ok(k3cuda_memcpy_h2d(ctx(), d, src, bytes), "upload");
    return d;
}

static void get(void *dst, const void *src, size_t bytes)
{
    ok(k3cuda_memcpy_d2h(ctx(), dst, src, bytes), "download");
    ok(k3cuda_sync(ctx()), "k3cuda_sync");
}

/* fp32 -> bf16, round to nearest even (bf16 is the top half of an fp32, k3.h k3_bf16f) */
static uint16_t bf16(float f)
{
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static uint16_t *to_bf16(const float *x, size_t n)
{
    uint16_t *h = (uint16_t *)malloc(n * sizeof(uint16_t) + 1);
    if (!h) {
        fprintf(stderr, "k3_gpu: FATAL, out of host memory\n");
        abort();
    }
    for (size_t i = 0; i < n; i++) h[i] = bf16(x[i]);
    return h;
}

void k3g_kda_step(float *S, float *o, const float *q, const float *k, const float *v,
                  const float *alpha, float beta, int dk, int dv)
{
    const size_t sb = (size_t)dk * dv * sizeof(float);
    float *dS = (float *)put(B_S, S, sb);
    void *dq = put(B_Q, q, (size_t)dk * 4), *dk_ = put(B_K, k, (size_t)dk * 4);
    void *dv_ = put(B_V, v, (size_t)dv * 4), *da = put(B_A, alpha, (size_t)dk * 4);
    void *db = put(B_B, &beta, 4);
    void *dO = dev(B_O, (size_t)dv * 4);
    ok(k3cuda_kda_decode(ctx(), dS, dO, dq, dk_, dv_, (const float *)da, (const float *)db, 1, 1,
                         dk, dv, 1.0f, K3CUDA_F32, K3CUDA_GATE_ALPHA),
       "k3cuda_kda_decode");
    get(S, dS, sb);
    get(o, dO, (size_t)dv * 4);
}

void k3g_kda_recurrence(float *S, float *o, const float *q, const float *k, const float *v,
                        const float *alpha, const float *beta, int T, int H, int D)
{
    if (T <= 0) return;
    const size_t P = (size_t)H * D, sb = (size_t)H * D * D * sizeof(float);
    const float qs = 1.0f / sqrtf((float)D);
    float *dS = (float *)dev(B_S, sb);
    if (S) ok(k3cuda_memcpy_h2d(ctx(), dS, S, sb), "upload state");
    else ok(k3cuda_memset(ctx(), dS, 0, sb), "zero state");
    char *dq = (char *)put(B_Q, q, (size_t)T * P * 4), *dk_ = (char *)put(B_K, k, (size_t)T * P * 4);
    char *dv_ = (char *)put(B_V, v, (size_t)T * P * 4);
    char *da = (char *)put(B_A, alpha, (size_t)T * P * 4);
    char *db = (char *)put(B_B, beta, (size_t)T * H * 4);
    char *dO = (char *)dev(B_O, (size_t)T * P * 4);
    if (T > 1 && (D == 64 || D == 128)) {
        int cu[2] = {0, T};
        size_t ws = 0;
        ok(k3cuda_kda_prefill_workspace(cu, 1, H, D, D, 64, &ws), "prefill workspace");
        void *dws = dev(B_WS, ws);
        ok(k3cuda_kda_prefill(ctx(), dS, dO, dq, dk_, dv_, (const float *)da, (const float *)db,
                              cu, 1, H, D, D, qs, K3CUDA_F32, K3CUDA_GATE_ALPHA, 64, dws, ws),
           "k3cuda_kda_prefill");
    } else {
        for (int t = 0; t < T; t++) {
            const size_t off = (size_t)t * P * 4;
            ok(k3cuda_kda_decode(ctx(), dS, dO + off, dq + off, dk_ + off, dv_ + off,
                                 (const float *)(da + off), (const float *)(db + (size_t)t * H * 4),
                                 1, H, D, D, qs, K3CUDA_F32, K3CUDA_GATE_ALPHA),
               "k3cuda_kda_decode");
        }
    }
    get(o, dO, (size_t)T * P * 4);
    if (S) get(S, dS, sb);
}

void k3g_mla_attend(float *acc, const float *q, const float *latent, const float *rope,
                    const float *kv_b, float scale, int H, int qn, int qr, int kv_lora, int vh,
                    int P)
{
    const int qh = qn + qr, kvd = qn + vh;
    uint16_t *hqn = to_bf16(q, (size_t)H * qh);      /* split below */
    uint16_t *hq_nope = (uint16_t *)malloc((size_t)H * qn * 2 + 1);
    uint16_t *hq_rope = (uint16_t *)malloc((size_t)H * qr * 2 + 1);
    uint16_t *hkvb = to_bf16(kv_b, (size_t)H * kvd * kv_lora);
    uint16_t *huk = (uint16_t *)malloc((size_t)H * qn * kv_lora * 2 + 1);
    uint16_t *huv = (uint16_t *)malloc((size_t)H * vh * kv_lora * 2 + 1);
    uint16_t *hlat = to_bf16(latent, (size_t)P * kv_lora);
    uint16_t *hrope = to_bf16(rope, (size_t)P * qr);
    if (!hq_nope || !hq_rope || !huk || !huv) {
        fprintf(stderr, "k3_gpu: FATAL, out of host memory\n");
        abort();
    }
    for (int h = 0; h < H; h++) {
        memcpy(hq_nope + (size_t)h * qn, hqn + (size_t)h * qh, (size_t)qn * 2);
        memcpy(hq_rope + (size_t)h * qr, hqn + (size_t)h * qh + qn, (size_t)qr * 2);
        memcpy(huk + (size_t)h * qn * kv_lora, hkvb + (size_t)h * kvd * kv_lora,
               (size_t)qn * kv_lora * 2);
        memcpy(huv + (size_t)h * vh * kv_lora, hkvb + ((size_t)h * kvd + qn) * kv_lora,
               (size_t)vh * kv_lora * 2);
    }
    void *dqn = put(B_QN, hq_nope, (size_t)H * qn * 2), *dqr = put(B_QR, hq_rope, (size_t)H * qr * 2);
    void *dlat = put(B_LAT, hlat, (size_t)P * kv_lora * 2), *drope = put(B_ROPE, hrope, (size_t)P * qr * 2);
    void *duk = put(B_UK, huk, (size_t)H * qn * kv_lora * 2);
    void *duv = put(B_UV, huv, (size_t)H * vh * kv_lora * 2);
    void *dO = dev(B_O, (size_t)H * vh * 4);
    int ctxlen = P;
    size_t ws = 0;
    ok(k3cuda_mla_decode_workspace(&ctxlen, 1, H, kv_lora, vh, &ws), "mla workspace");
    void *dws = dev(B_WS, ws);
    ok(k3cuda_mla_decode(ctx(), dO, K3CUDA_F32, dqn, dqr, dlat, drope, duk, duv, &ctxlen, 1, P, H,
                         qn, qr, kv_lora, vh, scale, dws, ws),
       "k3cuda_mla_decode");
    get(acc, dO, (size_t)H * vh * 4);
    free(hqn); free(hq_nope); free(hq_rope); free(hkvb); free(huk); free(huv);
    free(hlat); free(hrope);
}

/* Device copies of KDA layer weights, one allocation per layer, keyed by the host w->q. */
#define K3G_MAX_LAYERS 256
typedef struct {
    const void *key;
    void *block;
    k3cuda_kda_weights d;
} LayerW;
static LayerW g_lw[K3G_MAX_LAYERS];
static int g_nlw = 0;

static size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }

static const k3cuda_kda_weights *layer_weights(const k3g_kda_weights *w, int E, int H, int D,
                                               int K)
{
    for (int i = 0; i < g_nlw; i++)
        if (g_lw[i].key == w->q) return &g_lw[i].d;
    if (g_nlw == K3G_MAX_LAYERS) {
        fprintf(stderr, "k3_gpu: FATAL, more than %d KDA layers\n", K3G_MAX_LAYERS);
        abort();
    }
    const size_t P = (size_t)H * D, es = w->wdt == 1 ? 2 : 4;
    const void *src[14] = {w->q, w->k, w->v, w->q_conv, w->k_conv, w->v_conv, w->f_a, w->f_b,
                           w->A_log, w->dt_bias, w->b, w->g, w->o_norm, w->o};
    const size_t bytes[14] = {P * E * es, P * E * es, P * E * es, P * K * 4, P * K * 4,
                              P * K * 4, (size_t)D * E * es, P * D * es, (size_t)H * 4, P * 4,
                              (size_t)H * E * es, P * E * es, (size_t)D * 4, (size_t)E * P * es};
    size_t total = 0;
    for (int i = 0; i < 14; i++) total += a256(bytes[i]);
    LayerW *L = &g_lw[g_nlw];
    ok(k3cuda_malloc(ctx(), &L->block, total), "k3cuda_malloc (layer weights)");
    const void *dst[14];
    size_t off = 0;
    for (int i = 0; i < 14; i++) {
        if (!src[i]) {
            fprintf(stderr, "k3_gpu: FATAL, KDA layer weight %d is NULL\n", i);
            abort();
        }
        dst[i] = (char *)L->block + off;
        ok(k3cuda_memcpy_h2d(ctx(), (void *)dst[i], src[i], bytes[i]), "upload layer weights");
        off += a256(bytes[i]);
    }
    L->d.q = dst[0]; L->d.k = dst[1]; L->d.v = dst[2];
    L->d.q_conv = (const float *)dst[3]; L->d.k_conv = (const float *)dst[4];
    L->d.v_conv = (const float *)dst[5];
    L->d.f_a = dst[6]; L->d.f_b = dst[7];
    L->d.A_log = (const float *)dst[8]; L->d.dt_bias = (const float *)dst[9];
    L->d.b = dst[10]; L->d.g = dst[11]; L->d.o_norm = (const float *)dst[12]; L->d.o = dst[13];
    L->d.wdt = w->wdt == 1 ? K3CUDA_BF16 : K3CUDA_F32;
    L->key = w->q;
    g_nlw++;
    return &L->d;
}

void k3g_kda_layer(float *out, const float *x, const k3g_kda_weights *w, int T, int E, int H,
                   int D, int K, float gate_lb, float rms_eps, float *state)
{
    if (T <= 0) return;
    const k3cuda_kda_weights *dw = layer_weights(w, E, H, D, K);
    const size_t xb = (size_t)T * E * 4;
    const size_t sb = ((size_t)H * D * D + 3 * (size_t)H * D * (K - 1)) * 4;
    float *dx = (float *)put(B_Q, x, xb);
    float *dout = (float *)dev(B_O, xb);
    float *dS = NULL;
    if (state) dS = (float *)put(B_S, state, sb);
    size_t ws = 0;
    ok(k3cuda_kda_layer_workspace(T, E, H, D, K, dw->wdt, K3CUDA_F32, &ws), "layer workspace");
    void *dws = dev(B_WS, ws);
    ok(k3cuda_kda_layer(ctx(), dout, dx, dw, T, E, H, D, K, gate_lb, rms_eps, dS, K3CUDA_F32,
                        dws, ws),
       "k3cuda_kda_layer");
    get(out, dout, xb);
    if (state) get(state, dS, sb);
}

void k3g_shutdown(void)
{
    if (!g_ctx) return;
    for (int i = 0; i < g_nlw; i++) k3cuda_free(g_ctx, g_lw[i].block);
    g_nlw = 0;
    for (int i = 0; i < B_N; i++) {
        if (g_buf[i].ptr) k3cuda_free(g_ctx, g_buf[i].ptr);
        g_buf[i].ptr = NULL;
        g_buf[i].bytes = 0;
    }
    k3cuda_shutdown(g_ctx);
    g_ctx = NULL;
}
