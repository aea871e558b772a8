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

/* Release the process-wide context and staging buffers (optional, at exit). */
void k3g_shutdown(void);

#ifdef __cplusplus
}
#endif
#endif /* K3_GPU_H */
