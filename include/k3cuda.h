/* k3cuda.h -- libk3cuda: a B200 (sm_100a) attention engine for the kimi-k3-in-c C engine.
 *
 * Plain C ABI (extern "C", pointers and sizes, no C++ or framework types). Every entry
 * point returns an int status (K3CUDA_OK == 0) and never aborts; k3cuda_last_error()
 * gives the message of the most recent failure on the calling thread. The reference's
 * abort-on-failure contract (src/core/k3_ops.c:38-78) is kept one level up, by the C99
 * wrappers of include/k3_gpu.h.
 *
 * Device pointers ("d" in the comments) must come from k3cuda_malloc or any other CUDA
 * allocation on the context's device. All work is issued on the context's stream and is
 * asynchronous unless stated; k3cuda_sync waits for it.
 *
 * A context belongs to one host thread at a time: its stream, side streams, events and
 * staging ring are not locked. Threads that drive the GPU concurrently each create their
 * own context (the process-wide caches of tensor maps and kernel attributes are locked).
 *
 * Layouts follow the reference (include/k3/k3.h:157-165, src/core/k3_ops.c:864-938):
 *   per-token tensors      [tokens][heads][dim]       (the reference's [T][H*D])
 *   KDA recurrent state    [streams][heads][d_k][d_v] fp32, row = key channel
 *   MLA latent cache       [batch][cap][kv_lora] and rope cache [batch][cap][qk_rope]
 */
#ifndef K3CUDA_H
#define K3CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status codes */
enum {
    K3CUDA_OK = 0,
    K3CUDA_ERR_ARG = 1,         /* invalid argument (null pointer, bad size, misaligned) */
    K3CUDA_ERR_CUDA = 2,        /* a CUDA runtime call failed                              */
    K3CUDA_ERR_UNSUPPORTED = 3, /* shape or option this build has no kernel for            */
    K3CUDA_ERR_WORKSPACE = 4,   /* workspace smaller than the *_workspace query returned   */
    K3CUDA_ERR_NCCL = 5,        /* NCCL missing or a collective failed                     */
    K3CUDA_ERR_TIMEOUT = 6,     /* a bounded device-side wait gave up (error word set)     */
    K3CUDA_ERR_STATE = 7        /* call out of order (no communicator, context shut down)  */
};

/* element types of the per-token tensors */
enum { K3CUDA_F32 = 0, K3CUDA_BF16 = 1 };
/* gate semantics: log-decay g (alpha = exp(g), k3_ops.c:182) or alpha itself */
enum { K3CUDA_GATE_LOG = 0, K3CUDA_GATE_ALPHA = 1 };

typedef struct k3cuda_ctx k3cuda_ctx;

/* ------------------------------------------------------------ context and memory */
/* Create a context on `device` with its own non-blocking stream. */
int  k3cuda_init(int device, k3cuda_ctx **ctx);
/* Synchronise, release the stream, events, communicator and the context. */
int  k3cuda_shutdown(k3cuda_ctx *ctx);
/* Message of the last failure on this thread ("" when none). Never NULL. */
const char *k3cuda_last_error(void);
int  k3cuda_device_count(int *count);
/* Wait for all work issued on the context's stream. Returns K3CUDA_ERR_TIMEOUT when a
 * kernel's bounded device-side wait gave up (the kernel skipped its work and returned; the
 * context stays usable). With a communicator the wait runs under its deadline
 * (k3cuda_comm_set_timeout) and ends the communicator on a peer's failure. */
int  k3cuda_sync(k3cuda_ctx *ctx);
/* Bound of every device-side wait (mbarrier, peer flag) in this context's kernels, in SM
 * clock cycles; cycles <= 0 restores the default 2^31 (about a second at 1.9 GHz). A wait
 * that runs out records its code in the context's error word, the kernel drains its own
 * copies, frees its tensor memory and returns, and the next k3cuda_sync reports
 * K3CUDA_ERR_TIMEOUT. Applies to kernels launched after the call. */
int  k3cuda_set_wait_limit(k3cuda_ctx *ctx, long long cycles);
/* Launch one kernel that waits on a barrier nothing completes, under the bound above: the
 * timeout path (error word, K3CUDA_ERR_TIMEOUT from the next k3cuda_sync) exercised
 * without a fault, a trap or an unbounded spin. Takes as long as the bound. */
int  k3cuda_wait_selftest(k3cuda_ctx *ctx);
/* The context's cudaStream_t, as an opaque pointer (for callers that order their own
 * work against this library's). */
void *k3cuda_stream(k3cuda_ctx *ctx);
/* Device memory (256-byte aligned). */
int  k3cuda_malloc(k3cuda_ctx *ctx, void **dptr, size_t bytes);
int  k3cuda_free(k3cuda_ctx *ctx, void *dptr);
/* Page-locked host memory, for the host-buffer entry points' fast copies. */
int  k3cuda_host_alloc(k3cuda_ctx *ctx, void **hptr, size_t bytes);
int  k3cuda_host_free(k3cuda_ctx *ctx, void *hptr);
/* Copies on the context's stream (asynchronous for page-locked host memory). */
int  k3cuda_memcpy_h2d(k3cuda_ctx *ctx, void *dst, const void *src, size_t bytes);
int  k3cuda_memcpy_d2h(k3cuda_ctx *ctx, void *dst, const void *src, size_t bytes);
int  k3cuda_memcpy_d2d(k3cuda_ctx *ctx, void *dst, const void *src, size_t bytes);
int  k3cuda_memset(k3cuda_ctx *ctx, void *dptr, int value, size_t bytes);

/* ------------------------------------------------------------------------ timing */
/* Record event `slot` (0..K3CUDA_MAX_EVENTS-1) on the context's stream. */
#define K3CUDA_MAX_EVENTS 64
int  k3cuda_event_record(k3cuda_ctx *ctx, int slot);
/* Milliseconds between two recorded events (waits for the second). */
int  k3cuda_event_elapsed(k3cuda_ctx *ctx, int slot_a, int slot_b, float *ms);
/* Number of kernels this context has launched since init (all entry points). */
long long k3cuda_launch_count(k3cuda_ctx *ctx);
/* Zero-filled device buffer larger than L2, written once per call to evict L2 between
 * timed iterations (allocated on first use, freed at shutdown). */
int  k3cuda_flush_l2(k3cuda_ctx *ctx);

/* ------------------------------------------------------------- KDA decode (T = 1) */
/* One recurrent token for n_streams independent sequences x H heads. Replaces the
 * per-head call of k3_kda_step (src/core/k3_ops.c:186-243, contract include/k3/k3.h:
 * 157-165) that k3_kda_layer makes at T = 1 (k3_ops.c:927-938):
 *     S <- diag(alpha) S;  u = S^T k;  S <- S + k (beta (v - u))^T;  o = S^T q
 * with q multiplied by q_scale first (the reference pre-scales by d_k^-0.5,
 * k3_ops.c:918,934).
 *   state  d [n_streams][H][dk][dv] fp32, updated in place
 *   o      d [n_streams][H][dv]   io_dtype
 *   q, k   d [n_streams][H][dk]   io_dtype;   v d [n_streams][H][dv] io_dtype
 *   gate   d [n_streams][H][dk]   fp32, g (K3CUDA_GATE_LOG) or alpha (K3CUDA_GATE_ALPHA)
 *   beta   d [n_streams][H]       fp32
 * Fast path: dv == 128 and dk in {64, 128}; any other dk, dv <= 256 with
 * dk*dv <= 32768 runs a general kernel. */
int k3cuda_kda_decode(k3cuda_ctx *ctx, float *state, void *o, const void *q,
                      const void *k, const void *v, const float *gate, const float *beta,
                      int n_streams, int H, int dk, int dv, float q_scale, int io_dtype,
                      int gate_mode);

/* The same step with the per-token tensors in HOST memory and the state on the device
 * (the caller's view of k3_kda_step: token in, output back): o, q, k, v, gate, beta are
 * host pointers with k3cuda_kda_decode's layouts, state a device pointer. Two ways across
 * PCIe, chosen by `slices`:
 *   K3CUDA_HOST_IN_PLACE (-1): the buffers must be page-locked (k3cuda_host_alloc, which
 *       maps them into the device's address space); the kernel reads the inputs and writes
 *       o in place over PCIe: one launch, no copy, the transfer overlapping the step.
 *   0: chosen from the size: in place for small steps (up to 640 KB of inputs) when all
 *       six buffers are page-locked, else copies in one slice, or two from 4 MB up.
 *   1..K3CUDA_HOST_SLICES: copies through `staging`, the streams cut into that many batch
 *       slices; slice s's inputs come in on one copy stream while the kernel runs on slice
 *       s-1 and slice s-2's output goes back on another (a page-locked o is instead written
 *       by the kernels in place, with no copy back). Pageable memory works here but
 *       serialises the copies.
 * staging: a device buffer of k3cuda_kda_decode_host_workspace() bytes, 256-byte aligned
 * (may be NULL in place). Asynchronous like every entry point: o is complete when the
 * context's stream is (k3cuda_sync). */
#define K3CUDA_HOST_SLICES 16
#define K3CUDA_HOST_IN_PLACE (-1)
int k3cuda_kda_decode_host_workspace(int n_streams, int H, int dk, int dv, int io_dtype,
                                     size_t *bytes);
int k3cuda_kda_decode_host(k3cuda_ctx *ctx, float *state, void *o, const void *q,
                           const void *k, const void *v, const float *gate, const float *beta,
                           int n_streams, int H, int dk, int dv, float q_scale, int io_dtype,
                           int gate_mode, int slices, void *staging, size_t staging_bytes);

/* --------------------------------------------------- KDA chunked prefill (varlen) */
/* The whole recurrence of k3_kda_layer (src/core/k3_ops.c:908-938) over packed
 * variable-length sequences, computed chunkwise (WY / UT-transform form of the gated
 * delta rule) instead of token by token. Results equal the token-by-token recurrence to
 * floating-point rounding.
 *   cu_seqlens  HOST [n_seq + 1] token offsets into the packed tensors
 *   state       d [n_seq][H][dk][dv] fp32: initial state in, final state out; NULL
 *               means zero initial state and no state out
 *   o, q, k, v, gate, beta   as k3cuda_kda_decode, with [total_tokens] in place of
 *               [n_streams]
 *   chunk       64 (the only chunk size built)
 * Supported: dk == dv == 64 or 128. workspace must hold k3cuda_kda_prefill_workspace()
 * bytes (device memory, 256-byte aligned). Arithmetic: bf16 I/O at d = 128 runs on the
 * tensor cores with bf16 operands and fp32 accumulation; fp32 I/O at d = 128 runs its
 * chunk-local algebra in fp32 and the scan on the tensor cores with every operand split
 * into bf16 hi + lo (about 2^-16 relative error per product); d = 64 runs in fp32 on the
 * CUDA cores. */
int k3cuda_kda_prefill_workspace(const int *cu_seqlens, int n_seq, int H, int dk, int dv,
                                 int chunk, size_t *bytes);
int k3cuda_kda_prefill(k3cuda_ctx *ctx, float *state, void *o, const void *q,
                       const void *k, const void *v, const float *gate, const float *beta,
                       const int *cu_seqlens, int n_seq, int H, int dk, int dv,
                       float q_scale, int io_dtype, int gate_mode, int chunk,
                       void *workspace, size_t workspace_bytes);

/* Allocation-free k3cuda_kda_prefill. No counterpart in the reference (whose CPU kernels
 * need no device memory). It is for callers that cannot call cudaMalloc where they run a
 * prefill: a host runtime that has already reserved the whole HBM budget through its own
 * allocator, or a latency-critical path where cudaMalloc's implicit device synchronisation
 * would stall other streams. The workspace is a static device array of
 * K3CUDA_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until exit; a call
 * whose k3cuda_kda_prefill_workspace() size exceeds it fails with K3CUDA_ERR_WORKSPACE.
 * Arguments and results are those of k3cuda_kda_prefill. The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress); make that first call before any
 * stream capture. All calls share the one array and nothing in it needs to start zeroed
 * (every byte a call reads it has written first), but two calls whose kernels overlap on
 * the GPU (different streams or contexts on one device) race on it: serialise them. */
#define K3CUDA_NOALLOC_SCRATCH_BYTES (64u << 20)
int k3cuda_kda_prefill_noalloc(k3cuda_ctx *ctx, float *state, void *o, const void *q,
                               const void *k, const void *v, const float *gate,
                               const float *beta, const int *cu_seqlens, int n_seq, int H,
                               int dk, int dv, float q_scale, int io_dtype, int gate_mode,
                               int chunk);

/* ----------------------------------------------------------- MLA absorbed decode */
/* One query token per sequence over a compressed latent KV cache. Replaces the
 * attention loop of k3_mla_cached (src/core/k3_ops.c:381-411) at T = 1, with the
 * expanded per-head keys/values of the reference's cache (k3_ops.c:351-367) factored
 * through kv_b's per-head blocks W_UK = kv_b[h*(dn+dv) .. +dn) and
 * W_UV = kv_b[h*(dn+dv)+dn .. +dv):
 *     score[s] = (q_nope . (W_UK c_s) + q_rope . r_s) * scale
 *     out      = W_UV sum_s softmax(score)[s] c_s          (fp32 softmax)
 *   out       d [B][H][dv]     out_dtype (pre-gate accumulator acc of k3_ops.c:404-410)
 *   q_nope    d [B][H][dn] bf16;  q_rope d [B][H][dr] bf16
 *   latent    d [B][cap][dl] bf16; rope d [B][cap][dr] bf16
 *   w_uk      d [H][dn][dl] bf16;  w_uv d [H][dv][dl] bf16
 *   ctx_lens  HOST [B], 1 <= ctx_lens[b] <= cap: positions 0..ctx_lens[b]-1 attended
 * Supported: dn == dv == 128, dr == 64, dl == 512 (the released head geometry, k3.h
 * comments at :83-90), any H <= 128. */
int k3cuda_mla_decode_workspace(const int *ctx_lens, int B, int H, int dl, int dv,
                                size_t *bytes);
/* Host-only view of the attention work plan for B queries when the device offers
 * max_clusters two-SM clusters (a B200 offers 74): the number of (query, context range)
 * segments and of clusters it uses, and the workspace that exact plan needs at H = 128.
 * k3cuda_mla_decode_workspace returns a size that covers the plan for every cluster count,
 * so a buffer sized by it fits on any part. */
int k3cuda_mla_plan_stats(const int *ctx_lens, int B, int max_clusters, int *segments,
                          int *clusters, size_t *bytes);
int k3cuda_mla_decode(k3cuda_ctx *ctx, void *out, int out_dtype, const void *q_nope,
                      const void *q_rope, const void *latent, const void *rope,
                      const void *w_uk, const void *w_uv, const int *ctx_lens, int B,
                      int cap, int H, int dn, int dr, int dl, int dv, float scale,
                      void *workspace, size_t workspace_bytes);

/* The same attention with the query-to-cache map explicit: query b attends positions
 * [0, ctx_lens[b]) of cache sequence cache_seq[b] of a latent d [n_cache][cap][dl] / rope
 * d [n_cache][cap][dr] cache. A causal prefill chunk of T tokens at positions pos0 ..
 * pos0+T-1 of sequence s (after their rows are appended) is B = T queries with
 * cache_seq[b] = s and ctx_lens[b] = pos0 + b + 1: the attention of k3_mla_cached for
 * T > 1 (src/core/k3_ops.c:381-411, causal s <= p). k3cuda_mla_decode is the case
 * cache_seq[b] = b. cache_seq and ctx_lens are HOST arrays [B]; the workspace is
 * k3cuda_mla_decode_workspace(ctx_lens, B, ...). */
int k3cuda_mla_attend(k3cuda_ctx *ctx, void *out, int out_dtype, const void *q_nope,
                      const void *q_rope, const void *latent, const void *rope,
                      const void *w_uk, const void *w_uv, const int *cache_seq,
                      const int *ctx_lens, int B, int n_cache, int cap, int H, int dn, int dr,
                      int dl, int dv, float scale, void *workspace, size_t workspace_bytes);

/* Latent-cache append: the rows of T new tokens of sequence seq at positions pos0 ..
 * pos0+T-1, from the kv_a projection ct d [T][dl + dr] fp32 (k3_ops.c:363-366):
 *     latent[seq][pos0+t] = bf16(RMSNorm(ct[t][0:dl]) * kv_a_norm)   (norm over the latent
 *     rope[seq][pos0+t]   = bf16(ct[t][dl:dl+dr])                     only, eps = rms_eps)
 * latent d [n_cache][cap][dl] bf16, rope d [n_cache][cap][dr] bf16, kv_a_norm d [dl] fp32.
 * The reference expands each row through kv_b here; the absorbed attention above reads the
 * latent row instead. Supported: dl == 512, dr == 64. */
int k3cuda_mla_cache_append(k3cuda_ctx *ctx, void *latent, void *rope, const float *ct,
                            const float *kv_a_norm, float eps, int seq, int pos0, int T,
                            int n_cache, int cap, int dl, int dr);

/* ------------------------------------------------------- MLA layer forward */
/* Device weights of one MLA layer, field for field K3MlaW (include/k3/k3.h:203-210):
 * q_a [q_lora][E], q_b [H*(dn+dr)][q_lora], kv_a [dl+dr][E], kv_b [H*(dn+dv)][dl] (per head
 * dn W_UK rows then dv W_UV rows), o [E][H*dv], g [H*dv][E] or NULL (no gate), tagged by
 * wdt; q_a_norm [q_lora], kv_a_norm [dl] fp32. Every pointer is device memory. */
typedef struct {
    const void  *q_a, *q_b;
    const void  *kv_a, *kv_b;
    const void  *o, *g;
    const float *q_a_norm, *kv_a_norm;
    int          wdt;
} k3cuda_mla_weights;

/* k3_mla_cached (src/core/k3_ops.c:321-424) for T tokens of one sequence at positions
 * cached .. cached+T-1, with the cache on the device as the latent: latent d [cap][dl] bf16
 * and rope d [cap][dr] bf16 take the place of the reference's expanded kvc / ropec (the
 * layer writes the T new rows, then attends causally). out, x d [T][E] fp32. Attention
 * operands are bf16, accumulation fp32. Supported: the released geometry dn = 128, dr = 64,
 * dl = 512, dv = 128, H <= 128, E and q_lora multiples of 8, cached + T <= cap. workspace d:
 * k3cuda_mla_layer_workspace() bytes. */
int k3cuda_mla_layer_workspace(int T, int E, int H, int q_lora, int cached, int wdt,
                               size_t *bytes);
int k3cuda_mla_layer(k3cuda_ctx *ctx, float *out, const float *x, const k3cuda_mla_weights *w,
                     int T, int E, int H, int q_lora, int dn, int dr, int dl, int dv,
                     float rms_eps, void *latent, void *rope, int cached, int cap,
                     void *workspace, size_t workspace_bytes);

/* k3_mla_cached (src/core/k3_ops.c:321-424) for ANY head geometry -- the reference's own
 * test models use qk_nope 24, qk_rope 8, kv_lora 32, v_head 16 -- with an fp32 cache:
 * latent d [cap][dl] fp32 and rope d [cap][dr] fp32 (the layer writes the T new rows at
 * cached.., then attends causally). The attention is the absorbed form on CUDA cores in
 * fp32 (scores, softmax, accumulation), so results stay within fp32 rounding of the
 * reference instead of a bf16 bound; k3cuda_mla_layer is the tensor-core path for the
 * released geometry. Weights as k3cuda_mla_layer (fp32 or bf16 by wdt). Supported: E,
 * q_lora and H*dv multiples of 8, dl <= 1024, dr <= 256, cached + T <= cap. workspace d:
 * k3cuda_mla_layer_f32_workspace() bytes. */
int k3cuda_mla_layer_f32_workspace(int T, int E, int H, int q_lora, int dn, int dr, int dl,
                                   int dv, int wdt, size_t *bytes);
int k3cuda_mla_layer_f32(k3cuda_ctx *ctx, float *out, const float *x,
                         const k3cuda_mla_weights *w, int T, int E, int H, int q_lora, int dn,
                         int dr, int dl, int dv, float rms_eps, float *latent, float *rope,
                         int cached, int cap, void *workspace, size_t workspace_bytes);

/* ------------------------------------------------- multi-GPU: head-sharded output */
/* The reference is single-process (no communicator exists in it). Head sharding adds
 * one exchange: each rank computes H_local = H / nranks heads of [T][H][dv] and the
 * output is all-gathered over NVLink before o_proj. NCCL is loaded at run time
 * (libnccl.so.2); without it these return K3CUDA_ERR_NCCL. */
#define K3CUDA_UNIQUE_ID_BYTES 128
int k3cuda_comm_unique_id(unsigned char id[K3CUDA_UNIQUE_ID_BYTES]);
/* Collective. The communicator is non-blocking: every host wait on it (this call, the
 * fences of the gathered prefill, k3cuda_sync) polls NCCL's asynchronous error under a
 * deadline. A peer that leaves, stalls or fails ends the wait with ncclCommAbort and
 * K3CUDA_ERR_TIMEOUT or K3CUDA_ERR_NCCL, instead of a hang; afterwards the context's
 * single-GPU calls keep working and its collective calls return K3CUDA_ERR_STATE. */
int k3cuda_comm_init(k3cuda_ctx *ctx, int nranks, int rank,
                     const unsigned char id[K3CUDA_UNIQUE_ID_BYTES]);
/* Deadline of those waits in milliseconds (default 60000). */
int k3cuda_comm_set_timeout(k3cuda_ctx *ctx, int ms);
/* full d [T][nranks*H_local][dv] <- every rank's local d [T][H_local][dv] (rank r owns
 * heads r*H_local .. r*H_local+H_local-1). workspace d >= nranks*T*H_local*dv elements
 * of `dtype` (k3cuda_allgather_heads_workspace). */
int k3cuda_allgather_heads_workspace(int nranks, int T, int H_local, int dv, int dtype,
                                     size_t *bytes);
int k3cuda_allgather_heads(k3cuda_ctx *ctx, void *full, const void *local, int T,
                           int H_local, int dv, int dtype, void *workspace,
                           size_t workspace_bytes);

/* The prefill and the exchange in one call, without the all-gather's staging copy and
 * interleave pass: the head-sharded KDA prefill writes this rank's heads straight into
 * its own full [T][nranks*H_local][dv] bf16 buffer at their final place, and one
 * coalesced pass stores that head span into every peer's full buffer (peer memory over
 * NVLink, mapped by k3cuda_comm_register_full). It replaces k3cuda_kda_prefill +
 * k3cuda_allgather_heads at the head-sharded call site of k3_kda_layer
 * (src/core/k3_ops.c:908-949: recurrence, then the o_proj input).
 *
 * k3cuda_comm_register_full  collective (every rank, after k3cuda_comm_init): maps every
 *     rank's `full` (device memory from k3cuda_malloc/cudaMalloc, `bytes` long) into every
 *     process (CUDA IPC). Once per buffer; the mapping lives until k3cuda_shutdown.
 * k3cuda_kda_prefill_gathered  collective: arguments as k3cuda_kda_prefill with H_local
 *     heads per rank and no local output; bf16, dk == dv == 128. On return (in stream
 *     order) every rank's full buffer holds all heads: the call orders itself against the
 *     other ranks with two one-int all-reduces, before its writes and after them. */
#define K3CUDA_MAX_RANKS 8
int k3cuda_comm_register_full(k3cuda_ctx *ctx, void *full, size_t bytes);
int k3cuda_kda_prefill_gathered(k3cuda_ctx *ctx, float *state, const void *q, const void *k,
                                const void *v, const float *gate, const float *beta,
                                const int *cu_seqlens, int n_seq, int H_local, int dk,
                                int dv, float q_scale, int gate_mode, int chunk,
                                void *workspace, size_t workspace_bytes);

/* --------------------------------------------------- projections (k3_mmw on device) */
/* y d [T][out] fp32 = x d [T][in] fp32 times W d [out][in]^T, W fp32 (K3CUDA_F32) or bf16
 * (K3CUDA_BF16). The T-row form of k3_mmw (include/k3/k3.h:290-296: k3_matmul, k3_ops.c:
 * 265-291, and k3_matmul_bf16, :1122-1227, each one row). Products of the fp32 activation
 * and the weight are exact and summed in fp32 (the reference sums in double; the
 * difference is inside fp32 rounding of the result). T <= 8 streams every weight row once
 * (HBM-bound); T > 8 is a GEMM: for bf16 weights with in % 64 == 0 on tcgen05 with x split
 * into bf16 hi + lo halves (both halves' products accumulate in fp32, so the product keeps
 * near-fp32 accuracy), otherwise on the CUDA cores in fp32. Requires in % 8 == 0
 * and 16-byte aligned x, W, y. workspace d: k3cuda_matmul_workspace() bytes (0 when
 * T <= 8 or W is fp32). */
int k3cuda_matmul_workspace(int T, int in, int wdt, size_t *bytes);
int k3cuda_matmul(k3cuda_ctx *ctx, float *y, const float *x, const void *W, int wdt, int in,
                  int out, int T, void *workspace, size_t workspace_bytes);

/* ------------------------------------------------- MXFP4 expert projections */
/* The routed experts' weights in OCP MX FP4 (include/k3/k3.h:523-569): packed d
 * [rows][in/2] bytes, two E2M1 codes per byte, the LOW nibble the even element; scales d
 * [rows][in/group] E8M0 bytes; w = E2M1[code] * 2^(scale - 127), scale 255 read as 0.
 *
 * k3cuda_mxfp4_dequant replaces k3_mxfp4_dequant (src/core/k3_ops.c:1801-1831): out d
 * [rows][in] fp32 or bf16 (both exact). k3cuda_matmul_mxfp4 replaces k3_matmul_mxfp4
 * (:1394-1799) for T activation rows: y d [T][rows] fp32 = x d [T][in] fp32 times W^T,
 * never materialising W when T <= 4, group == 32 and in % 32 == 0 (products exact, each
 * 32-element group summed in fp32 then scaled, groups summed in fp32); otherwise W is
 * expanded to bf16 in the workspace and multiplied on tcgen05 against x's bf16 hi + lo
 * halves. Requirements of the reference: in even, group <= 64. */
int k3cuda_mxfp4_dequant(k3cuda_ctx *ctx, void *out, int out_dtype,
                         const unsigned char *packed, const unsigned char *scales, int rows,
                         int in, int group);
int k3cuda_matmul_mxfp4_workspace(int T, int in, int rows, int group, size_t *bytes);
int k3cuda_matmul_mxfp4(k3cuda_ctx *ctx, float *y, const float *x, const unsigned char *packed,
                        const unsigned char *scales, int in, int rows, int group, int T,
                        void *workspace, size_t workspace_bytes);
/* n (<= 64) matrices of one shape in one launch, each with its own x and y: the decode
 * step of k3_moe (k3_ops.c:640-645), where every selected expert's w1 and w3 multiply the
 * same z, or each expert's w2 its own activation. HOST arrays of device pointers; group
 * 32, T <= 4, in % 32 == 0. */
int k3cuda_matmul_mxfp4_batch(k3cuda_ctx *ctx, float *const *y, const float *const *x,
                              const unsigned char *const *packed,
                              const unsigned char *const *scales, int n, int in, int rows,
                              int T);

/* --------------------------------------------------------- KDA layer forward */
/* Device weights of one KDA layer, field for field K3KdaW (include/k3/k3.h:449-463):
 * q, k, v, g [H*D][E], f_a [D][E], f_b [H*D][D], b [H][E], o [E][H*D] are tagged by wdt
 * (K3CUDA_F32 == K3_WF32, K3CUDA_BF16 == K3_WBF16); the conv kernels [H*D][K], A_log [H],
 * dt_bias [H*D] and o_norm [D] are fp32. Every pointer is device memory. */
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
} k3cuda_kda_weights;

/* k3_kda_layer (src/core/k3_ops.c:864-951) for one sequence of T tokens, every activation
 * on the device: projections, ShortConv + SiLU with the carried history, L2 on q and k,
 * beta, the decay chain, the recurrence (the decode kernel at T == 1, the chunked prefill
 * at T > 1 for D in {64, 128}, else the decode kernel once per token), head RMSNorm, the
 * sigmoid gate and o_proj, in the reference's order.
 *   out    d [T][E] fp32;  x d [T][E] fp32
 *   state  d [H*D*D + 3*H*D*(K-1)] fp32 (recurrent state, then the q, k, v conv
 *          histories), updated in place; NULL = fresh sequence, nothing written back
 *   io_dtype  the recurrence's q, k, v and output type: K3CUDA_BF16 runs the prefill on
 *          the tensor cores (D == 128), K3CUDA_F32 keeps every operand fp32
 * Supported: E % 8 == 0, D % 16 == 0, D <= 128, 1 <= K <= 4. workspace d:
 * k3cuda_kda_layer_workspace() bytes, 256-byte aligned. */
int k3cuda_kda_layer_workspace(int T, int E, int H, int D, int K, int wdt, int io_dtype,
                               size_t *bytes);
int k3cuda_kda_layer(k3cuda_ctx *ctx, float *out, const float *x,
                     const k3cuda_kda_weights *w, int T, int E, int H, int D, int K,
                     float gate_lb, float rms_eps, float *state, int io_dtype,
                     void *workspace, size_t workspace_bytes);

#ifdef __cplusplus
}
#endif
#endif /* K3CUDA_H */
