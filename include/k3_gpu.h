/* k3_gpu.h -- C99 drop-ins for the kimi-k3-in-c attention hot path, run on a B200.
 *
 * Each function keeps the argument meaning, layout and error behaviour of the reference
 * code it replaces, on host fp32 buffers, so a caller of the reference can switch by
 * renaming the call. Internally they stage the buffers to the device and call
 * libk3cuda (include/k3cuda.h). Like the reference (src/core/k3_ops.c:38-78) they return
 * void and abort with a message on any failure rather than leave an output unwritten.
 * Not thread-safe: the reference's caller is single-threaded (k3_run.c:1096-1109). The
 * device is K3CUDA_DEVICE from the environment, else 0.
 */
#ifndef K3_GPU_H
#define K3_GPU_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Replaces k3_kda_step (include/k3/k3.h:157-165, src/core/k3_ops.c:186-243): one head,
 * one token, S [dk][dv] updated in place, q already scaled by d_k^-0.5. */
void k3g_kda_step(float *S, float *o, const float *q, const float *k, const float *v,
                  const float *alpha, float beta, int dk, int dv);

/* Replaces the recurrence block of k3_kda_layer (src/core/k3_ops.c:908-938): all H heads
 * over T tokens. S [H][D][D] in place (NULL: zero state, as k3_ops.c:911-917);
 * q, k, v, alpha, o [T][H*D]; beta [T][H]. q is scaled by 1/sqrt(D) here, as
 * k3_ops.c:918,934 does. T == 1 runs the decode kernel, T > 1 the chunked prefill
 * (D in {64, 128}) or, for other D, the decode kernel once per token. */
void k3g_kda_recurrence(float *S, float *o, const float *q, const float *k, const float *v,
                        const float *alpha, const float *beta, int T, int H, int D);

/* Replaces the attention loop of k3_mla_cached (src/core/k3_ops.c:381-411) for one query
 * token attending positions 0..P-1, over a LATENT cache instead of the expanded one:
 *   acc    [H][vh]            out: the pre-gate accumulator (k3_ops.c:404-410)
 *   q      [H][qn + qr]       the token's query row, as k3_ops.c:357 forms it
 *   latent [P][kv_lora]       kv_a_norm(kv_a x)[:kv_lora] per position (k3_ops.c:363-365)
 *   rope   [P][qr]            the shared rope slot per position (k3_ops.c:366)
 *   kv_b   [H*(qn+vh)][kv_lora]  the reference's weight; rows h*(qn+vh).. are W_UK[h],
 *                                the next vh rows W_UV[h] (k3_ops.c:367,391,408)
 * scale is (qn+qr)^-0.5 (k3_ops.c:328). Inputs are rounded to bf16 on the device. */
void k3g_mla_attend(float *acc, const float *q, const float *latent, const float *rope,
                    const float *kv_b, float scale, int H, int qn, int qr, int kv_lora,
                    int vh, int P);

/* Host weights of one KDA layer, field for field K3KdaW (include/k3/k3.h:449-463): same
 * order, same types, so a K3KdaW pointer can be passed by cast. wdt: 0 fp32, 1 bf16. */
typedef struct {
    const void  *q, *k, *v;
    const float *q_conv, *k_conv, *v_conv;
    const void  *f_a, *f_b;
    const float *A_log;
    const float *dt_bias;
    const void  *b;
    const void  *g;
    const float *o_norm;
    const void  *o;
    int          wdt;
} k3g_kda_weights;

/* Replaces k3_kda_layer (src/core/k3_ops.c:864-951) for host buffers: out, x [T][E]; state
 * [H*D*D + 3*H*D*(K-1)] updated in place (NULL: fresh sequence, as the reference). E, H, D,
 * K, gate_lb and rms_eps are the K3Cfg fields hidden, kda_heads, kda_head_dim, conv_k,
 * gate_lb and rms_eps. The recurrence runs on fp32 operands. The layer's weights are copied
 * to the device on the first call that sees them (keyed by the address of w->q) and kept
 * until k3g_shutdown: the reference never changes a loaded layer's weights. A caller that
 * frees a layer and loads another (whose q may land at the same address) calls
 * k3g_shutdown in between. */
void k3g_kda_layer(float *out, const float *x, const k3g_kda_weights *w, int T, int E, int H,
                   int D, int K, float gate_lb, float rms_eps, float *state);

/* State file for device-resident state (--save-state / --load-state of the reference,
 * src/cli/k3_state.c:102-270). The header is the reference's K3StateHdr byte for byte
 * (magic "K3ST", then version, config fingerprint, counts, per-layer geometry, FNV-1a
 * payload hash over the header with the hash zeroed and then the payload), with version
 * K3G_STATE_VER: the reference's loader refuses it by version rather than misreading it.
 * What changes is the MLA part: the device keeps the latent cache, so kvpp is the latent
 * width (kv_lora) and ropepp the rope width, and those slices are bf16.
 *   payload: seq [nseq] int32; ks [n_bound][kper] fp32; latent [n_mla][cached][kv_lora]
 *            bf16; rope [n_mla][cached][rope_w] bf16 (position-major per layer, only the
 *            occupied positions, so a resumed run may size its cache differently)
 *   device:  ks d [n_bound][kper]; latent d [n_mla][kv_cap][kv_lora]; rope d
 *            [n_mla][kv_cap][rope_w]
 * fp is the reference's 12-int config fingerprint (k3_state_fp). Both return 0, or -1
 * with a message on stderr (the reference's contract): save writes a temporary file
 * beside `path`, fsyncs it and renames it over `path`; load refuses a file of another
 * version, architecture (fp), geometry, layer count or capacity, a truncated or longer
 * file, or one whose hash does not match. On load *nseq and *cached receive the counts
 * and seq must hold seq_cap ints. */
#define K3G_STATE_VER 4
int k3g_state_save(const char *path, const int32_t fp[12], const int *seq, int nseq,
                   const float *d_ks, int64_t kper, int n_bound, const void *d_latent,
                   const void *d_rope, int n_mla, int kv_cap, int kv_lora, int rope_w,
                   int cached);
int k3g_state_load(const char *path, const int32_t fp[12], int *seq, int seq_cap, int *nseq,
                   float *d_ks, int64_t kper, int n_bound, void *d_latent, void *d_rope,
                   int n_mla, int kv_cap, int kv_lora, int rope_w, int *cached);

/* Release the process-wide context, staging buffers and cached weights (optional, at exit). */
void k3g_shutdown(void);

#ifdef __cplusplus
}
#endif
#endif /* K3_GPU_H */
