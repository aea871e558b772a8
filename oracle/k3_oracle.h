/* k3_oracle.h -- CPU restatement of the kimi-k3-in-c attention hot path.
 *
 * TEST INFRASTRUCTURE, NOT PRODUCT CODE. Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference legs load this library, and only as the checker.
 * The CUDA library (libk3cuda) never links or calls it.
 *
 * Every function restates one piece of the reference engine (FareedKhan-dev/kimi-k3-in-c)
 * and names the reference file:line it follows. Parity is pinned twice:
 *   1. against the reference's own fixtures (tests/fixtures/ops/kda_recur{1,8}.json,
 *      kda_decay.json, kda_layer{1,8}.json, mla.json), converted to tests/golden/*.npz;
 *   2. against the reference C itself, compiled unmodified into oracle/_ref/libk3ref.so.
 *
 * Layouts follow the reference: per token [T][H][d] row-major (the reference's [T][H*D]),
 * recurrent state [H][d_k][d_v] row-major with row = key channel (include/k3/k3.h:157-165).
 */
#ifndef K3_ORACLE_H
#define K3_ORACLE_H

#ifdef __cplusplus
extern "C" {
#endif

/* k3_kda_step, src/core/k3_ops.c:186-243. One head, one token, q pre-scaled. */
void orc_kda_step(float *S, float *o, const float *q, const float *k, const float *v,
                  const float *alpha, float beta, int dk, int dv);

/* The recurrence driver of k3_kda_layer, src/core/k3_ops.c:908-938, generalised to
 * packed variable-length sequences (cu_seqlens[nseq+1], token offsets).
 *   S     [nseq][H][dk][dv] in/out; NULL means zero initial state and no state out
 *   o     [sum T][H][dv]
 *   q,k   [sum T][H][dk], v [sum T][H][dv]
 *   gate  [sum T][H][dk]: log-decay g (gate_is_log=1, alpha = expf(g), as
 *         k3_ops.c:182) or alpha itself (gate_is_log=0)
 *   beta  [sum T][H]
 * q is multiplied by q_scale before each step (k3_ops.c:918,934). Heads and sequences
 * run on up to nthreads OpenMP threads; every head keeps its serial order in t. */
void orc_kda_recurrence(float *S, float *o, const float *q, const float *k,
                        const float *v, const float *gate, int gate_is_log,
                        const float *beta, const int *cu_seqlens, int nseq, int H,
                        int dk, int dv, float q_scale, int nthreads);

/* k3_kda_decay, src/core/k3_ops.c:167-183 (A_log indexed per head). */
void orc_kda_decay(float *g, float *alpha, const float *z, const float *A_log,
                   const float *dt_bias, int H, int D, float lb);

/* k3_rmsnorm, src/core/k3_ops.c:94-101 (double accumulator, eps inside the sqrt). */
void orc_rmsnorm(float *y, const float *x, const float *w, int n, float eps);

/* l2norm_, src/core/k3_ops.c:845-851 (sum of squares, not mean). */
void orc_l2norm(float *v, int n, float eps);

/* k3_shortconv, src/core/k3_ops.c:133-165 (causal depthwise conv + SiLU, state in place). */
void orc_shortconv(float *y, const float *x, const float *w, float *state,
                   int channels, int k, int T);

/* k3_kda_layer, src/core/k3_ops.c:864-951, fp32 weights only (K3_WF32).
 * Weight shapes as K3KdaW (include/k3/k3.h:448-462). state as k3.h:465-467:
 * H*D*D recurrent floats then 3*H*D*(conv_k-1) conv floats; NULL = fresh sequence. */
void orc_kda_layer(float *out, const float *x, int T, int hidden, int H, int D,
                   int conv_k, float gate_lb, float rms_eps,
                   const float *Wq, const float *Wk, const float *Wv,
                   const float *q_conv, const float *k_conv, const float *v_conv,
                   const float *f_a, const float *f_b, const float *A_log,
                   const float *dt_bias, const float *Wb, const float *Wg,
                   const float *o_norm, const float *Wo, float *state);

/* Absorbed MLA decode: the attention loop of k3_mla_cached (src/core/k3_ops.c:381-411)
 * for ONE query token per sequence at position ctx_len-1, restated over the latent
 * cache with the expanded keys/values factored as k_nope = W_UK c, v = W_UV c
 * (kv_b rows [h*256, h*256+128) and [h*256+128, h*256+256), k3_ops.c:367,391,408).
 *   out    [B][H][dv]      pre-gate attention output (acc in k3_ops.c:404-410)
 *   q_nope [B][H][dn], q_rope [B][H][dr]
 *   latent [B][cap][dl], rope [B][cap][dr]   (positions 0..ctx_lens[b]-1 attended)
 *   w_uk   [H][dn][dl], w_uv [H][dv][dl]
 * Score dots and the softmax sum accumulate in double, exp is expf, as the reference. */
void orc_mla_absorbed_decode(float *out, const float *q_nope, const float *q_rope,
                             const float *latent, const float *rope,
                             const float *w_uk, const float *w_uv,
                             const int *ctx_lens, int B, int cap, int H, int dn,
                             int dr, int dl, int dv, float scale, int nthreads);

/* Chunkwise (WY / UT-transform) restatement of the same recurrence, in double, used to
 * produce the intra-chunk known-answer vectors the reference does not have
 * (include/k3/k3.h:51-60 says the reference never forms them). One head, one
 * sequence, zero initial state, T a multiple of C. Writes per chunk n:
 *   Akk [n][C][C] strictly lower  beta_t * (k_t . k_s) * prod_{s<u<=t} alpha_u
 *   Aqk [n][C][C] lower incl diag (q_t . k_s) * prod_{s<u<=t} alpha_u     (q scaled)
 *   o   [T][dv], S [dk][dv] final state.
 * It must agree with orc_kda_recurrence; the tests check that it does. */
void orc_kda_chunked_f64(float *o, float *S, double *Akk, double *Aqk,
                         const float *q, const float *k, const float *v,
                         const float *g, const float *beta, int T, int C, int dk,
                         int dv, float q_scale);

/* MXFP4 (OCP MX FP4, include/k3/k3.h:523-569): packed [rows][in/2] bytes, the LOW nibble
 * the even element; scales [rows][in/group] E8M0 bytes; value = E2M1[nibble] *
 * 2^(scale - 127), scale 255 read as 0. k3_mxfp4_dequant (src/core/k3_ops.c:1801-1831). */
void orc_mxfp4_dequant(float *out, const unsigned char *packed, const unsigned char *scales,
                       int rows, int in, int group);

/* y[t][r] = sum_i W[r][i] x[t][i] with W read as MXFP4, every product and the row sum in
 * double: the arithmetic k3_matmul_mxfp4 (src/core/k3_ops.c:1394-1799) is held to (its
 * test: dequantise-then-matmul within 1e-6 relative). */
void orc_matmul_mxfp4(float *y, const float *x, const unsigned char *packed,
                      const unsigned char *scales, int in, int rows, int T, int group);

#ifdef __cplusplus
}
#endif
#endif /* K3_ORACLE_H */
