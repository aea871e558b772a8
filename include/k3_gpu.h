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

/* Model configuration, field for field K3Cfg (include/k3/k3.h:73-120): same order, same
 * types, so a K3Cfg pointer can be passed by cast. The drop-ins read hidden and rms_eps, the
 * KDA fields (kda_heads, kda_head_dim, conv_k, gate_lb) and the MLA fields (n_heads, q_lora,
 * kv_lora, qk_nope, qk_rope, v_head). */
typedef struct {
    int   hidden, n_layers, vocab;
    float rms_eps;
    int   kda_heads, kda_head_dim, conv_k;
    float gate_lb;
    int   n_heads, q_lora, kv_lora, qk_nope, qk_rope, v_head, mla_out_gate;
    int   n_experts, topk, n_shared, latent, moe_inter;
    float routed_scale;
    int   moe_renorm, latent_norm;
    int   first_dense, dense_inter;
    int   attn_res_block;
    float situ_b1, situ_b2;
    int   n_full_attn;
    int  *full_attn;
} k3g_cfg;

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

/* Host weights of one MLA layer, field for field K3MlaW (include/k3/k3.h:203-210); g may be
 * NULL (no output gate). */
typedef struct {
    const void  *q_a, *q_b;
    const void  *kv_a, *kv_b;
    const void  *o, *g;
    const float *q_a_norm, *kv_a_norm;
    int          wdt;
} k3g_mla_weights;

/* Replaces k3_kda_layer (include/k3/k3.h:468-469, src/core/k3_ops.c:864-951), same
 * signature: out, x [T][hidden]; state [H*D*D + 3*H*D*(conv_k-1)] updated in place (NULL:
 * a fresh sequence, nothing kept, as the reference). scratch is accepted and not touched
 * (the device work uses device workspaces), so a buffer sized by k3_kda_scratch may be
 * passed as before. The recurrence runs on fp32 operands. The layer's weights are copied to
 * the device on the first call that sees them and reused while the same host arrays come
 * back: the copy is keyed by the address of w->q, the layer geometry and wdt, and a
 * fingerprint of sampled bytes of every weight array, so a layer freed and another loaded
 * at the same address is noticed and copied again. */
void k3g_kda_layer(float *out, const float *x, const k3g_kda_weights *w, const k3g_cfg *c,
                   int T, float *state, float *scratch);

/* Replaces k3_mla_cached (include/k3/k3.h:219-221, src/core/k3_ops.c:321-424), same
 * signature and contract: T tokens at positions cached .. cached+T-1 of one sequence;
 * kvc [cap][n_heads*(qk_nope+v_head)] and ropec [cap][qk_rope] carry the cache between calls
 * (kvc == NULL: no cache, the T tokens attend among themselves, as k3_mla); a position at or
 * past cap aborts with the reference's message (k3_ops.c:333-334). scratch is accepted and
 * not touched.
 * The cache lives on the device as the compressed latent: bf16 rows with the tensor-core
 * attention at the released head geometry (qk_nope 128, qk_rope 64, kv_lora 512, v_head
 * 128), fp32 rows with the fp32 CUDA-core attention for any other geometry (or everywhere
 * with K3G_MLA_F32=1 in the environment). The host buffers stay the record of the cache, in
 * the latent form: row p of kvc holds position p's normalised latent (its first kv_lora
 * floats, exactly the device row widened to fp32; the rest of the row is not written), and
 * row p of ropec its rope slot, as the reference stores it. So kvc must be at least kv_lora
 * floats wide, and a cache written by these drop-ins is not the reference's expanded form
 * (do not hand one to the CPU k3_mla_cached, or the reverse). The device copy is keyed by
 * kvc: rows the device does not hold (a copied or reloaded buffer, a new kvc) are uploaded
 * from the host rows before the call. The last row before `cached` is checked against what
 * the device holds; a caller that rewrites earlier rows of the same buffer in place calls
 * k3g_mla_cache_forget(kvc) first. */
void k3g_mla_cached(float *out, const float *x, const k3g_mla_weights *w, const k3g_cfg *c,
                    int T, float *scratch, float *kvc, float *ropec, int cached, int cap);
/* Drop the device copy of the cache whose host rows are kvc (the next call re-uploads). */
void k3g_mla_cache_forget(const float *kvc);

/* Both layer drop-ins honour K3G_TOKENWISE=1 in the environment: a call of T > 1 tokens
 * runs as T consecutive one-token calls. Results then do not depend on how a sequence is
 * cut into calls -- the property the reference's prefix-reuse gate demands bit for bit
 * (tests/unit/k3_model.c:431-441) -- at the cost of prefill speed (no chunked recurrence,
 * no GEMM projections). By default a multi-token call runs the chunked prefill and GEMMs,
 * equal to the token-by-token result within the stated tolerance, not bit for bit. */

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
