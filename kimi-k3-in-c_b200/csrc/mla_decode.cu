// mla_decode.cu -- absorbed MLA decode over the compressed latent cache, on tcgen05.
//
// Replaces the per-head attention loop of k3_mla_cached (reference src/core/k3_ops.c:
// 381-411) for one query token per sequence. The reference caches the EXPANDED keys and
// values (k3_ops.c:304-315, 351-367); here the cache holds the latent c_s (512 wide) and the
// shared rope slot r_s (64), and the per-head blocks of kv_b are folded into the query and
// the output:
//     q_lat = W_UK^T q_nope                       mla_q_absorb_tc   (tcgen05, bf16 [B][128][576])
//     S     = [q_lat | q_rope] . [c_s | r_s]^T    mla_attend_tc     (tcgen05, fp32 in TMEM)
//     P     = softmax(S * scale)                  mla_attend_tc     (fp32 on CUDA cores)
//     o_lat = P . C                               mla_attend_tc     (tcgen05, fp32 in TMEM)
//     merge the context splits                    mla_merge         (flash-decoding identity)
//     out   = W_UV o_lat                          mla_project_tc    (tcgen05)
//
// mla_attend_tc runs as clusters of two CTAs (one SM each). All 128 heads are the MMA's M.
// The 576-wide contraction of S is split across the pair -- rank 0 takes latent dims
// [0,256) and the 64 rope dims, rank 1 latent dims [256,512) -- and each rank accumulates
// the output for its own 256 latent dims, which are exactly the dims whose tiles it already
// holds. Per 64-token tile each rank computes its partial S, sends it to the peer with
// asynchronous cluster stores that complete on the peer's mbarrier (no fences on the path),
// both add the two partials in the same order (rank 0's + rank 1's), so both derive the same
// softmax, and each multiplies P by its half of the tile. Per SM:
//   TMEM    S 64 columns + this rank's query half (160 columns, the MMA's A operand read
//           straight from TMEM) + O 256 columns                                     (of 512)
//   shared  3 KV stages x 40 KB + 2 P x 16 KB + 2 exchange x 32 KB                 (~217 KB)
// Keeping the query in TMEM leaves shared memory to the KV pipeline. P and the exchange
// buffers are double-buffered so that the softmax of tile g overlaps the P.V product of
// tile g-1.
// Warp roles: warp 0 issues TMA loads; warp 1 allocates TMEM and issues S = Q.K^T; warp 10
// issues O += P.V; warps 2-9 (two threads per head = TMEM lane, 32 score columns each) write
// the query into TMEM, run the exchange, the softmax and the epilogue; the two threads of a
// head combine their row max and row sum through an mbarrier of the warp pair. The running
// max is only moved when it grows by more than 2^8 (a lazy rescale: numerator and
// denominator use the same stale max, so the result is exact), which keeps the O rescale in
// TMEM off the common path. The score exchange of tile g overlaps the softmax of tile g-1:
// tile g's partial is sent first, then tile g-1 is finished.
//
// Work: the (sequence, 64-token tile) list is cut into equal contiguous ranges, one per
// cluster; a range that crosses sequences becomes several segments, each writing a partial
// (max, sum, o_lat) per head; mla_merge combines the segments of every sequence (the
// flash-decoding identity) and mla_project_tc applies W_UV.
//
// Every wait is bounded (sm100.cuh): on a timeout the kernel records an error word, skips
// the rest of its work, waits briefly for its own loads and frees TMEM; k3cuda_sync then
// reports K3CUDA_ERR_TIMEOUT.
#include <string.h>

#include <algorithm>
#include <vector>

#include "internal.cuh"
#include "sm100.cuh"
#include "tmap.cuh"

namespace k3 {

using namespace sm100;

constexpr int MLA_DN = 128, MLA_DR = 64, MLA_DL = 512, MLA_DV = 128;
constexpr int MLA_QW = MLA_DL + MLA_DR;    // 576: absorbed query width
constexpr int MLA_HP = 128;                // heads padded to the MMA's M
constexpr int MLA_TILE = 64;               // tokens per tile
constexpr int MLA_MIN_TILES = 4;           // fewest tiles the work plan gives a cluster
// A segment's fixed work (query load into TMEM, pipeline drain, partial write-out) in tile
// units, for the work plan. Measured on a 4096-token causal prefill (per-step median):
// 0 (tiles only) 10.34 ms, 3: 7.37, 6: 6.56, 8: 6.65, 10: 6.74.
constexpr int MLA_SEG_COST = 6;
constexpr int MLA_PF = 6;                  // tiles the L2 prefetch runs ahead of the loads
constexpr int MLA_NST = 3;                 // KV pipeline stages
constexpr int MLA_KVBLK = MLA_TILE * 128;  // bytes of one 64-dim block of a KV tile
constexpr int MLA_NBLK = 5;                // dim blocks of rank 0 (4 latent + rope); rank 1: 4
constexpr int MLA_OFF_KV = 0;
constexpr int MLA_OFF_P = MLA_OFF_KV + MLA_NST * MLA_NBLK * MLA_KVBLK;
constexpr int MLA_PBUF = MLA_HP * 128;     // one P buffer: 128 rows x 128 B (K-major, SW128)
constexpr int MLA_OFF_X = MLA_OFF_P + 2 * MLA_PBUF;
constexpr int MLA_XBUF = MLA_HP * MLA_TILE * 4;  // one exchange buffer: 128 heads x 64 fp32
constexpr int MLA_SMEM = MLA_OFF_X + 2 * MLA_XBUF + 1024;  // + alignment slack
static_assert(MLA_KVBLK % 1024 == 0 && MLA_OFF_P % 1024 == 0 && MLA_PBUF % 1024 == 0,
              "swizzled operands need 1024-byte alignment");
constexpr int MLA_PART = MLA_DL + 4;       // floats per (segment, head): o_lat, max, sum, pad
                                           // (rows stay 16-byte aligned for float4 stores)
// TMEM columns: S [0, 64), this rank's query half [64, 224) (two bf16 per column),
// O [256, 512)
constexpr int MLA_TM_S = 0, MLA_TM_Q = 64, MLA_TM_O = 256, MLA_TM_COLS = 512;
constexpr float MLA_RESCALE_LOG2 = 8.f;    // lazy rescale threshold (factor 256)

__device__ __forceinline__ float bf(const __nv_bfloat16 *p) { return __bfloat162float(*p); }

// A bounded wait taken by a whole warp: every lane waits, and the result is the AND over
// the warp, so warp-collective TMEM instructions after it run converged.
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity, unsigned *err,
                                          unsigned code, bool cluster_scope = false) {
    const bool ok = cluster_scope ? mbar_wait_cluster(bar, parity, err, code)
                                  : mbar_wait(bar, parity, err, code);
    return __all_sync(0xffffffffu, ok);
}

// ------------------------------------------------------------------ per-head GEMMs
// The two small per-head products around the attention, on tcgen05 with the sequences as the
// MMA's M (128 per CTA; rows past B are zero-filled by TMA and never stored):
//   mla_q_absorb_tc  qlat[b][h][0:512] = q_nope[b][h] (1 x 128) . W_UK[h] (128 x 512), bf16,
//                    and qlat[b][h][512:576] = q_rope[b][h]; two CTAs per head (256 columns)
//   mla_project_tc   out[b][h][:] = o_lat[b][h] (1 x 512) . W_UV[h]^T (512 x 128), with
//                    o_lat carried as a bf16 hi/lo pair (K = 1024, W_UV's blocks read twice)
//                    so the fp32 o_lat reaches the MMA to ~16 mantissa bits
struct HeadGemmMaps {
    CUtensorMap a, b;
};

// CTA (h, y, z) computes columns [256 z, +256) of q_lat for 128 sequences: a head's 128 KB
// W_UK block is split over two CTAs, and two CTAs (97 KB of shared memory each) share an SM.
__global__ void __launch_bounds__(128, 2)
mla_q_absorb_tc(const __grid_constant__ HeadGemmMaps maps, const __nv_bfloat16 *__restrict__ q_rope,
                __nv_bfloat16 *__restrict__ qlat, int B, int H, unsigned *__restrict__ err) {
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    uint8_t *sA = sm;              // 2 K-blocks x [128 b][128 B]
    uint8_t *sB = sm + 2 * 16384;  // [2 K-blocks][4 N-blocks] x [64 i][128 B]
    __shared__ uint64_t bar_ld, bar_mma;
    __shared__ uint32_t tslot;
    const int h = blockIdx.x, b0 = blockIdx.y * 128, z = blockIdx.z, tid = threadIdx.x,
              warp = tid >> 5;
    if (tid == 0) {
        mbar_init(&bar_ld, 1);
        mbar_init(&bar_mma, 1);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(&tslot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = tslot;
    if (tid == 0) {
        mbar_expect_tx(&bar_ld, 2 * 16384 + 8 * 8192);
        for (int kb = 0; kb < 2; kb++) tma_load_3d(sA + kb * 16384, &maps.a, &bar_ld, kb * 64, h, b0);
        for (int kb = 0; kb < 2; kb++)
            for (int nb = 0; nb < 4; nb++)
                tma_load_3d(sB + (kb * 4 + nb) * 8192, &maps.b, &bar_ld, (4 * z + nb) * 64, kb * 64,
                            h);
        if (mbar_wait(&bar_ld, 0, err, 0x401)) {
            tc_fence_after();
            constexpr uint32_t id = idesc_f16(128, 256, false, true);
            for (int ks = 0; ks < 8; ks++) {
                const int kb = ks / 4, kin = ks % 4;
                const uint64_t ad = sdesc_kmajor(smem_u32(sA + kb * 16384 + kin * 32));
                const uint64_t bd = sdesc_mnmajor(smem_u32(sB + kb * 4 * 8192 + kin * 2048), 8192);
                mma_bf16_ss(tb, ad, bd, id, ks ? 1u : 0u);
            }
            mma_commit(&bar_mma);
        }
    }
    __syncwarp();
    const bool ok = warp_wait(&bar_mma, 0, err, 0x402);
    tc_fence_after();
    const int b = b0 + 32 * warp + (tid & 31);
    if (ok) {
        for (int c = 0; c < 256; c += 16) {
            float v[16];
            tmem_ld16(tb + ((uint32_t)(32 * warp) << 16) + c, v);
            tmem_wait_ld();
            if (b < B) {
                uint32_t pk[8];
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const __nv_bfloat162 t2 = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
                    pk[i] = *reinterpret_cast<const uint32_t *>(&t2);
                }
                uint4 *dst = reinterpret_cast<uint4 *>(qlat + ((size_t)b * MLA_HP + h) * MLA_QW +
                                                       256 * z + c);
                dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            }
        }
        if (b < B && z == 0) {
            const uint4 *src = reinterpret_cast<const uint4 *>(q_rope + ((size_t)b * H + h) * MLA_DR);
            uint4 *dst = reinterpret_cast<uint4 *>(qlat + ((size_t)b * MLA_HP + h) * MLA_QW + MLA_DL);
#pragma unroll
            for (int i = 0; i < MLA_DR / 8; i++) dst[i] = src[i];
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tb, 256);
    }
}

template <typename OUT>
__global__ void __launch_bounds__(128, 2)
mla_project_tc(const __grid_constant__ HeadGemmMaps maps, OUT *__restrict__ out, int B, int H,
               unsigned *__restrict__ err) {
    // K blocks of 64 (hi 0..7, lo 8..15); each stage holds one A block (o_lat rows) and the
    // W_UV block it meets, so a CTA needs 97 KB of shared memory and two share an SM
    constexpr int NS = 3, KB = 16, STAGE = 2 * 16384;
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    __shared__ uint64_t bar_full[NS], bar_empty[NS], bar_mma;
    __shared__ uint32_t tslot;
    const int h = blockIdx.x, b0 = blockIdx.y * 128, tid = threadIdx.x, warp = tid >> 5;
    if (tid == 0) {
        mbar_init(&bar_mma, 1);
        for (int i = 0; i < NS; i++) {
            mbar_init(&bar_full[i], 1);
            mbar_init(&bar_empty[i], 1);
        }
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(&tslot, 128);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tb = tslot;
    if (tid == 0) {
        auto load = [&](int kb) {  // block kb into stage kb % NS
            uint8_t *st = sm + (kb % NS) * STAGE;
            mbar_expect_tx(&bar_full[kb % NS], STAGE);
            tma_load_3d(st, &maps.a, &bar_full[kb % NS], kb * 64, h, b0);
            tma_load_3d(st + 16384, &maps.b, &bar_full[kb % NS], (kb % 8) * 64, 0, h);
        };
        for (int kb = 0; kb < NS; kb++) load(kb);
        bool ok = true;
        constexpr uint32_t id = idesc_f16(128, 128, false, false);
        for (int kb = 0; kb < KB && ok; kb++) {
            const int st = kb % NS;
            if (!(ok = mbar_wait(&bar_full[st], (kb / NS) & 1, err, 0x412))) break;
            tc_fence_after();
            for (int kin = 0; kin < 4; kin++) {
                const uint64_t ad = sdesc_kmajor(smem_u32(sm + st * STAGE + kin * 32));
                const uint64_t bd = sdesc_kmajor(smem_u32(sm + st * STAGE + 16384 + kin * 32));
                mma_bf16_ss(tb, ad, bd, id, (kb | kin) ? 1u : 0u);
            }
            mma_commit(&bar_empty[st]);
            // refill the previous block's stage while this block's MMAs run
            const int pk = kb - 1;
            if (pk >= 0 && pk + NS < KB) {
                if (!(ok = mbar_wait(&bar_empty[pk % NS], (pk / NS) & 1, err, 0x413))) break;
                load(pk + NS);
            }
        }
        if (ok) mma_commit(&bar_mma);
        // drain: the last load of every stage has landed before the CTA may exit
        for (int st = 0; st < NS; st++) {
            const int jl = st + NS * ((KB - 1 - st) / NS);  // the last block of stage st
            mbar_wait_quiet(&bar_full[st], (jl / NS) & 1);
        }
    }
    __syncwarp();
    const bool ok = warp_wait(&bar_mma, 0, err, 0x414);
    tc_fence_after();
    const int b = b0 + 32 * warp + (tid & 31);
    if (ok) {
        for (int c = 0; c < 128; c += 16) {
            float v[16];
            tmem_ld16(tb + ((uint32_t)(32 * warp) << 16) + c, v);
            tmem_wait_ld();
            if (b < B)
#pragma unroll
                for (int i = 0; i < 16; i++) io<OUT>::st(out + ((size_t)b * H + h) * MLA_DV + c + i, v[i]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tb, 128);
    }
}

// ---------------------------------------------------------------------------- attend
struct MlaSeg {
    int b, t0, t1, slot;  // sequence, tile range [t0, t1), partial slot
};

struct MlaMaps {
    CUtensorMap lat, rope;
};

struct MlaBars {
    uint64_t kv_full[MLA_NST], kv_empty[MLA_NST];
    uint64_t q_full, q_empty;
    uint64_t s_full[2], s_empty[2];
    uint64_t p_full[2], pv_done[2];
    uint64_t x_full[2], x_empty[2];
    uint64_t pair[4];           // per lane quarter: the two softmax warps of those rows
    float pair_val[2][2][128];  // [phase parity][column half][head]
    uint32_t tmem_base;
};

constexpr int MLA_THREADS = 352;  // 11 warps: TMA, S issuer, 8 softmax, PV issuer
constexpr int MLA_SOFT = 256;     // softmax threads: two per head (32 score columns each)

__global__ void __launch_bounds__(MLA_THREADS, 1) __cluster_dims__(2, 1, 1)
mla_attend_tc(const __grid_constant__ MlaMaps maps, const MlaSeg *__restrict__ segs,
              const int *__restrict__ cl_begin, const int *__restrict__ ctx_lens,
              const __nv_bfloat16 *__restrict__ qlat, float *__restrict__ part, int H,
              const int *__restrict__ row0, float scale_log2e, unsigned *__restrict__ err) {
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    __shared__ MlaBars bars;
    pdl_trigger();
    pdl_wait();  // the work plan, q_lat and the cache come from earlier work
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t rank = cluster_rank(), peer = rank ^ 1u;
    const int cl = blockIdx.x >> 1;
    const int sbeg = cl_begin[cl], send = cl_begin[cl + 1];
    const int nblk = rank == 0 ? 5 : 4;
    const int dim0 = rank == 0 ? 0 : 256;  // first latent dim of this rank

    if (tid == 0) {
        for (int s = 0; s < MLA_NST; s++) {
            mbar_init(&bars.kv_full[s], 1);
            mbar_init(&bars.kv_empty[s], 1);
        }
        mbar_init(&bars.q_full, MLA_SOFT);
        mbar_init(&bars.q_empty, 1);
        for (int s = 0; s < 2; s++) {
            mbar_init(&bars.s_full[s], 1);
            mbar_init(&bars.s_empty[s], MLA_SOFT);
            mbar_init(&bars.p_full[s], MLA_SOFT);
            mbar_init(&bars.pv_done[s], 1);
            mbar_init(&bars.x_full[s], 1);
            mbar_init(&bars.x_empty[s], 8);  // one arrive per softmax warp of the peer
        }
        for (int q = 0; q < 4; q++) mbar_init(&bars.pair[q], 64);
        fence_barrier_init();
    }
    if (warp == 1) tmem_alloc(&bars.tmem_base, MLA_TM_COLS);
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // barrier init visible to the peer before any remote arrive
    tc_fence_after();
    const uint32_t tbase = bars.tmem_base;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            prefetch_tmap(&maps.lat);
            prefetch_tmap(&maps.rope);
            int g = 0;
            int last_use[MLA_NST];
            for (int st = 0; st < MLA_NST; st++) last_use[st] = -1;
            bool ok = true;
            // L2 prefetch cursor: MLA_PF tiles ahead of the tile being loaded. A stage is
            // only refilled after its tile's P.V, so without it every load pays the full
            // HBM latency on the critical path (measured: the score issuer waited ~2200
            // cycles per tile for its data); the prefetched rows arrive from L2 instead.
            int pf_si = sbeg, pf_t = sbeg < send ? segs[sbeg].t0 : 0;
            auto pf_next = [&]() {  // prefetch the cursor's tile and advance it
                if (pf_si >= send) return;
                const MlaSeg ps = segs[pf_si];
                const int prow = row0[ps.b] + pf_t * MLA_TILE;
                for (int kb = 0; kb < 4; kb++) tma_prefetch_2d(&maps.lat, dim0 + kb * 64, prow);
                if (nblk == 5) tma_prefetch_2d(&maps.rope, 0, prow);
                if (++pf_t >= ps.t1 && ++pf_si < send) pf_t = segs[pf_si].t0;
            };
            for (int i = 0; i < MLA_PF; i++) pf_next();  // the cursor starts MLA_PF tiles ahead
            for (int si = sbeg; si < send && ok; si++) {
                const MlaSeg sg = segs[si];
                for (int t = sg.t0; t < sg.t1; t++, g++) {
                    const int st = g % MLA_NST, n = g / MLA_NST;
                    pf_next();
                    if (n > 0 && !(ok = mbar_wait(&bars.kv_empty[st], (n - 1) & 1, err, 0x102)))
                        break;
                    mbar_expect_tx(&bars.kv_full[st], nblk * MLA_KVBLK);
                    uint8_t *dst = sm + MLA_OFF_KV + st * MLA_NBLK * MLA_KVBLK;
                    const int row = row0[sg.b] + t * MLA_TILE;
                    for (int kb = 0; kb < 4; kb++)
                        tma_load_2d(dst + kb * MLA_KVBLK, &maps.lat, &bars.kv_full[st],
                                    dim0 + kb * 64, row);
                    if (nblk == 5)
                        tma_load_2d(dst + 4 * MLA_KVBLK, &maps.rope, &bars.kv_full[st], 0, row);
                    last_use[st] = n;
                }
            }
            // loads still in flight are waited for (bounded) before the CTA may exit
            for (int st = 0; st < MLA_NST; st++)
                if (last_use[st] >= 0) mbar_wait_quiet(&bars.kv_full[st], last_use[st] & 1);
        }
    } else if (warp == 1) {
        // ------------------------------------------------- S issuer: S = Q . K^T
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_f16(128, MLA_TILE, false, false);
            int g = 0, nq = 0, prev_b = -1;
            bool ok = true;
            for (int si = sbeg; si < send && ok; si++) {
                const MlaSeg sg = segs[si];
                const bool qlast = si + 1 >= send || segs[si + 1].b != sg.b;
                if (sg.b != prev_b) {  // the softmax warps have written this batch's Q
                    if (!(ok = mbar_wait(&bars.q_full, nq & 1, err, 0x201))) break;
                    nq++;
                    prev_b = sg.b;
                }
                for (int t = sg.t0; t < sg.t1 && ok; t++, g++) {
                    const int st = g % MLA_NST, sb = 0;
                    if (!(ok = mbar_wait(&bars.kv_full[st], (g / MLA_NST) & 1, err, 0x202))) break;
                    if (g >= 1 && !(ok = mbar_wait(&bars.s_empty[0], (g - 1) & 1, err, 0x204)))
                        break;
                    tc_fence_after();
                    const uint8_t *kv = sm + MLA_OFF_KV + st * MLA_NBLK * MLA_KVBLK;
                    for (int kb = 0; kb < nblk; kb++)
#pragma unroll
                        for (int ks = 0; ks < 4; ks++)
                            mma_bf16_ts(tbase + MLA_TM_S + sb * MLA_TILE,
                                        tbase + MLA_TM_Q + kb * 32 + ks * 8,
                                        sdesc_kmajor(smem_u32(kv + kb * MLA_KVBLK + ks * 32)), id_s,
                                        (kb | ks) ? 1u : 0u);
                    mma_commit(&bars.s_full[sb]);
                    if (qlast && t + 1 == sg.t1) mma_commit(&bars.q_empty);
                }
            }
        }
    } else if (warp == 10) {
        // ------------------------------------------ PV issuer: O (+)= P . V_half
        if (lane == 0) {
            constexpr uint32_t id_o = idesc_f16(128, 256, false, true);
            int g = 0;
            for (int si = sbeg; si < send; si++) {
                const MlaSeg sg = segs[si];
                bool ok = true;
                for (int t = sg.t0; t < sg.t1; t++, g++) {
                    if (!(ok = mbar_wait(&bars.p_full[g & 1], (g >> 1) & 1, err, 0x203))) break;
                    tc_fence_after();
                    const uint8_t *kv = sm + MLA_OFF_KV + (g % MLA_NST) * MLA_NBLK * MLA_KVBLK;
                    const uint8_t *P = sm + MLA_OFF_P + (g & 1) * MLA_PBUF;
#pragma unroll
                    for (int ks = 0; ks < MLA_TILE / 16; ks++)
                        mma_bf16_ss(tbase + MLA_TM_O, sdesc_kmajor(smem_u32(P + ks * 32)),
                                    sdesc_mnmajor(smem_u32(kv + ks * 2048), MLA_KVBLK), id_o,
                                    (t == sg.t0 && ks == 0) ? 0u : 1u);
                    mma_commit(&bars.kv_empty[g % MLA_NST]);
                    mma_commit(&bars.pv_done[g & 1]);
                }
                if (!ok) break;
            }
        }
    } else {
        // ------------------------------------- Q load, exchange, softmax, epilogue
        // Two warps per lane quarter: warp 2 + q and warp 6 + q own heads 32 q .. 32 q + 31
        // (TMEM lanes) and score columns [32 hc, 32 hc + 32) of every tile; the row max and
        // the row sum are combined through the pair's mbarrier.
        const int q4 = warp & 3, hc = (warp - 2) >> 2, sw = warp - 2;
        const int row = 32 * q4 + lane;  // head == TMEM lane
        const int c0 = 32 * hc;          // first score column of this thread
        const uint32_t lane_off = (uint32_t)(32 * q4) << 16;
        const uint32_t xpeer = map_peer(smem_u32(sm + MLA_OFF_X), peer);
        float m_ref = -INFINITY, l = 0.f;  // l: this thread's half of the row sum
        int g = 0, cur_slot = -1, nq = 0, prev_b = -1, np = 0;
        bool ok = true;
        // the partner warp's value for this row (bounded wait on the pair's mbarrier); both
        // warps of a pair call this at the same points, so their phases stay in step
        auto pair_value = [&](float v, bool &good) -> float {
            bars.pair_val[np & 1][hc][row] = v;
            mbar_arrive(&bars.pair[q4]);
            good = warp_wait(&bars.pair[q4], np & 1, err, 0x30a) && good;
            const float o = bars.pair_val[np & 1][hc ^ 1][row];
            np++;
            return o;
        };
        auto epilogue = [&](int slot) -> bool {  // warp-collective: every lane loads its row
            bool good = true;
            const float lt = l + pair_value(l, good);
            float *dst = part + ((size_t)slot * H + row) * MLA_PART;
            for (int c = 128 * hc; c < 128 * hc + 128; c += 16) {
                float v[16];
                tmem_ld16(tbase + lane_off + MLA_TM_O + c, v);
                tmem_wait_ld();
                if (row < H) {
                    float4 *d4 = reinterpret_cast<float4 *>(dst + rank * 256 + c);
#pragma unroll
                    for (int i = 0; i < 4; i++)
                        d4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
                }
            }
            if (rank == 0 && hc == 0 && row < H) {
                dst[MLA_DL] = m_ref;
                dst[MLA_DL + 1] = lt;
            }
            return good;
        };
        // Tiles are handled with a one-tile skew: tile g's partial scores are sent to the
        // peer, then tile g-1 -- whose peer partial arrived meanwhile -- is finished (softmax,
        // P). The exchange latency overlaps the next tile's score read-out.
        struct Pending {
            int g, valid, slot;
            bool newseg;
        };
        constexpr int HT = MLA_TILE / 2;  // score columns per thread
        float sp[HT];  // this rank's partial scores of the pending tile (this thread's columns)
        Pending pd{-1, 0, -1, false};
        auto finish = [&](const Pending &q) -> bool {
            const int xb = q.g & 1, pb = q.g & 1;
            if (!warp_wait(&bars.x_full[xb], (q.g >> 1) & 1, err, 0x303, true)) return false;
            const float4 *X4 = reinterpret_cast<const float4 *>(sm + MLA_OFF_X + xb * MLA_XBUF);
            float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
            for (int i = 0; i < HT / 4; i++) {
                const float4 o = X4[(c0 / 4 + i) * MLA_HP + row];
                const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int c = 4 * i + j;
                    const float tot = rank == 0 ? sp[c] + ov[j] : ov[j] + sp[c];
                    sp[c] = c0 + c < q.valid ? tot * scale_log2e : -INFINITY;
                    m4[j] = fmaxf(m4[j], sp[c]);
                }
            }
            // this warp's part of exchange buffer xb is read (the values are consumed above):
            // lane 0 tells the peer that it may be refilled
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster_relaxed(&bars.x_empty[xb], peer);
            bool good = true;
            float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
            mx = fmaxf(mx, pair_value(mx, good));
            if (!good) return false;
            if (q.newseg) {
                // a new segment: the previous segment's last P.V must be done before its O is
                // read out and the next P.V overwrites it
                if (q.g > 0) {
                    if (!warp_wait(&bars.pv_done[(q.g - 1) & 1], ((q.g - 1) >> 1) & 1, err, 0x304))
                        return false;
                    tc_fence_after();
                }
                if (cur_slot >= 0 && !epilogue(cur_slot)) return false;
                cur_slot = q.slot;
                m_ref = mx;
                l = 0.f;
            } else {
                const bool grow = mx > m_ref + MLA_RESCALE_LOG2;
                if (__any_sync(0xffffffffu, grow)) {
                    // O is rescaled in place: the previous tile's P.V must be done
                    if (!warp_wait(&bars.pv_done[(q.g - 1) & 1], ((q.g - 1) >> 1) & 1, err, 0x306))
                        return false;
                    tc_fence_after();
                    const float f = grow ? exp2f(m_ref - mx) : 1.f;
                    for (int c = 128 * hc; c < 128 * hc + 128; c += 16) {
                        float v[16];
                        tmem_ld16(tbase + lane_off + MLA_TM_O + c, v);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; i++) v[i] *= f;
                        tmem_st16(tbase + lane_off + MLA_TM_O + c, v);
                    }
                    tmem_wait_st();
                    if (grow) {
                        l *= f;
                        m_ref = mx;
                    }
                }
            }
            // P buffer pb is free once the P.V of tile g-2 is done
            uint8_t *P = sm + MLA_OFF_P + pb * MLA_PBUF;
            if (q.g >= 2 && !warp_wait(&bars.pv_done[pb], ((q.g >> 1) - 1) & 1, err, 0x307))
                return false;
            // P row (bf16, 128-byte swizzle: 16-byte chunk c of row r sits at c ^ (r & 7))
            float rs[4] = {0.f, 0.f, 0.f, 0.f};
            uint32_t pk[HT / 2];
#pragma unroll
            for (int c = 0; c < HT; c += 2) {
                const float p0 = ex2_approx(sp[c] - m_ref), p1 = ex2_approx(sp[c + 1] - m_ref);
                rs[(c >> 1) & 3] += p0 + p1;
                const __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
                pk[c / 2] = *reinterpret_cast<const uint32_t *>(&h2);
            }
            l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
#pragma unroll
            for (int c = 0; c < HT / 8; c++) {
                const int ch = c0 / 8 + c;  // 16-byte chunk of the 128-byte P row
                *reinterpret_cast<uint4 *>(P + row * 128 + ((ch ^ (row & 7)) * 16)) =
                    make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            }
            if (q.valid < MLA_TILE) {
                // rows past the context may hold anything (even NaN): zero this rank's value
                // rows there so that P = 0 times them stays 0
                uint8_t *kv = sm + MLA_OFF_KV + (q.g % MLA_NST) * MLA_NBLK * MLA_KVBLK;
                const int nz = (MLA_TILE - q.valid) * 8;  // 16-byte chunks per block
                for (int e = 32 * sw + lane; e < 4 * nz; e += MLA_SOFT) {
                    const int kb = e / nz, r = q.valid + (e % nz) / 8, c = e % 8;
                    *reinterpret_cast<uint4 *>(kv + kb * MLA_KVBLK + r * 128 + c * 16) =
                        make_uint4(0, 0, 0, 0);
                }
            }
            fence_async_shared();
            tc_fence_before();
            mbar_arrive(&bars.p_full[pb]);
            return true;
        };
        for (int si = sbeg; si < send && ok; si++) {
            const MlaSeg sg = segs[si];
            const int clen = ctx_lens[sg.b];
            if (sg.b != prev_b) {
                // this rank's query half into TMEM (lane = head, two bf16 per column): the
                // previous batch's S products must be done with the old one
                if (nq > 0 && !(ok = warp_wait(&bars.q_empty, (nq - 1) & 1, err, 0x308))) break;
                tc_fence_after();
                const uint4 *qrow =
                    reinterpret_cast<const uint4 *>(qlat + ((size_t)sg.b * MLA_HP + row) * MLA_QW);
                for (int kb = 0; kb < nblk; kb++) {
                    const int d0 = kb < 4 ? dim0 + kb * 64 : MLA_DL;  // first dim of block
                    float v[16];  // this warp's 32 dims of the block (16 columns)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const uint4 w = qrow[(d0 + hc * 32) / 8 + i];
                        v[4 * i] = __uint_as_float(w.x);
                        v[4 * i + 1] = __uint_as_float(w.y);
                        v[4 * i + 2] = __uint_as_float(w.z);
                        v[4 * i + 3] = __uint_as_float(w.w);
                    }
                    tmem_st16(tbase + lane_off + MLA_TM_Q + kb * 32 + hc * 16, v);
                }
                tmem_wait_st();
                tc_fence_before();
                mbar_arrive(&bars.q_full);
                nq++;
                prev_b = sg.b;
            }
            for (int t = sg.t0; t < sg.t1; t++, g++) {
                const int xb = g & 1;
                if (sw == 0 && lane == 0) mbar_expect_tx(&bars.x_full[xb], MLA_XBUF);
                float s[HT];
                if (!(ok = warp_wait(&bars.s_full[0], g & 1, err, 0x301))) break;
                tc_fence_after();
                tmem_ld32(tbase + lane_off + MLA_TM_S + c0, s);
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(&bars.s_empty[0]);
                // send this thread's partial scores into the peer's exchange buffer xb
                // (X4[i * 128 + row] = float4 i of `row`); the transfer completes on the
                // peer's x_full[xb]
                if (g >= 2 &&
                    !(ok = warp_wait(&bars.x_empty[xb], ((g >> 1) - 1) & 1, err, 0x302, true)))
                    break;
                const uint32_t rbar = map_peer(smem_u32(&bars.x_full[xb]), peer);
#pragma unroll
                for (int i = 0; i < HT / 4; i++)
                    st_async_v4(xpeer + (uint32_t)(xb * MLA_XBUF + ((c0 / 4 + i) * MLA_HP + row) * 16),
                                s[4 * i], s[4 * i + 1], s[4 * i + 2], s[4 * i + 3], rbar);
                if (pd.g >= 0 && !(ok = finish(pd))) break;
#pragma unroll
                for (int c = 0; c < HT; c++) sp[c] = s[c];
                pd = Pending{g, clen - t * MLA_TILE, sg.slot, t == sg.t0};
            }
        }
        if (ok && pd.g >= 0) ok = finish(pd);
        if (ok && g > 0 &&
            warp_wait(&bars.pv_done[(g - 1) & 1], ((g - 1) >> 1) & 1, err, 0x305)) {
            tc_fence_after();
            epilogue(cur_slot);
        }
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer no longer writes into this CTA's shared memory
    if (warp == 1) {
        __syncwarp();
        tmem_dealloc(tbase, MLA_TM_COLS);
    }
}

// ------------------------------------------------- per-head products for a few sequences
// With B <= MLA_SMALL_B sequences the tcgen05 kernels above run one CTA per head whose time
// is the latency of streaming its 128 KB weight block through one SM. These spread each
// head's block over several CTAs instead, every thread issuing all its 16-byte weight loads
// before any arithmetic, with fp32 accumulation on the CUDA cores.
constexpr int MLA_SMALL_B = 8;

// qlat[b][h][c] = sum_i q_nope[b][h][i] W_UK[h][i][c] (bf16 out) for the 128 columns
// c in [128 z, +128) of CTA (h, z); z == 0 also copies q_rope into qlat[b][h][512:576].
// Thread t: columns 128 z + 8 (t % 16) .. +8, rows i = t / 16 + 16 j (j < 8). NB >= B is
// the register budget for the sequences.
template <int NB>
__global__ void __launch_bounds__(256)
mla_q_absorb_small(const __nv_bfloat16 *__restrict__ q_nope,
                   const __nv_bfloat16 *__restrict__ q_rope, const __nv_bfloat16 *__restrict__ w_uk,
                   long long uk_head_elems, __nv_bfloat16 *__restrict__ qlat, int B, int H) {
    __shared__ float qs[NB][MLA_DN];
    __shared__ float red[8][NB][128];
    pdl_trigger();
    const int h = blockIdx.x, z = blockIdx.y, tid = threadIdx.x, warp = tid >> 5;
    const int cg = tid & 15, r0 = tid >> 4, c0 = 128 * z + 8 * cg;
    uint4 wv[8];
    if (h < H) {
        const __nv_bfloat16 *W = w_uk + (size_t)h * uk_head_elems + c0;
#pragma unroll
        for (int j = 0; j < 8; j++)
            wv[j] = __ldg(reinterpret_cast<const uint4 *>(W + (size_t)(r0 + 16 * j) * MLA_DL));
    }
    pdl_wait();  // the weights above are never written by the chain; q_nope is
    if (h >= H) {
        // a padding head of the MMA's M: its query row must score zero
        for (int e = tid; e < B * 128; e += 256)
            qlat[((size_t)(e >> 7) * MLA_HP + h) * MLA_QW + 128 * z + (e & 127)] =
                __float2bfloat16_rn(0.f);
        if (z == 0)
            for (int e = tid; e < B * MLA_DR; e += 256)
                qlat[((size_t)(e / MLA_DR) * MLA_HP + h) * MLA_QW + MLA_DL + e % MLA_DR] =
                    __float2bfloat16_rn(0.f);
        return;
    }
    for (int e = tid; e < NB * MLA_DN; e += 256) {
        const int b = e / MLA_DN, i = e % MLA_DN;
        qs[b][i] = b < B ? __bfloat162float(q_nope[((size_t)b * H + h) * MLA_DN + i]) : 0.f;
    }
    __syncthreads();
    float acc[NB][8];
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
        for (int x = 0; x < 8; x++) acc[b][x] = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const uint32_t u[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
        float wf[8];
#pragma unroll
        for (int x = 0; x < 4; x++) {
            wf[2 * x] = __uint_as_float(u[x] << 16);
            wf[2 * x + 1] = __uint_as_float(u[x] & 0xffff0000u);
        }
#pragma unroll
        for (int b = 0; b < NB; b++) {
            const float qv = qs[b][r0 + 16 * j];
#pragma unroll
            for (int x = 0; x < 8; x++) acc[b][x] = fmaf(qv, wf[x], acc[b][x]);
        }
    }
    // the two row sets of a warp (lanes l and l + 16) first, then the eight warps
#pragma unroll
    for (int b = 0; b < NB; b++)
#pragma unroll
        for (int x = 0; x < 8; x++) acc[b][x] += __shfl_xor_sync(0xffffffffu, acc[b][x], 16);
    if ((tid & 31) < 16) {
#pragma unroll
        for (int b = 0; b < NB; b++)
#pragma unroll
            for (int x = 0; x < 8; x++) red[warp][b][8 * cg + x] = acc[b][x];
    }
    __syncthreads();
    for (int e = tid; e < B * 128; e += 256) {
        const int b = e >> 7, c = e & 127;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < 8; w++) v += red[w][b][c];
        qlat[((size_t)b * MLA_HP + h) * MLA_QW + 128 * z + c] = __float2bfloat16_rn(v);
    }
    if (z == 0)
        for (int e = tid; e < B * MLA_DR; e += 256)
            qlat[((size_t)(e / MLA_DR) * MLA_HP + h) * MLA_QW + MLA_DL + e % MLA_DR] =
                q_rope[((size_t)(e / MLA_DR) * H + h) * MLA_DR + e % MLA_DR];
}

// out[b][h][j] = sum_k o_lat[b][h][k] W_UV[h][j][k] for the 16 rows j in [16 z, +16) of
// CTA (h, z), o_lat = hi + lo of the merge's bf16 pair. Warp w: rows 16 z + 2 w, +1; lane:
// k in [16 lane, +16).
template <typename OUT>
__global__ void __launch_bounds__(256)
mla_project_small(const __nv_bfloat16 *__restrict__ olat2, const __nv_bfloat16 *__restrict__ w_uv,
                  long long uv_head_elems, OUT *__restrict__ out, int B, int H) {
    // o_lat rows with one pad float after every 16: lane l reads elements 16 l .. 16 l + 15,
    // at 17 l .. 17 l + 15, so the 32 lanes of a read fall in 32 different banks
    constexpr int OSW = MLA_DL + MLA_DL / 16;
    __shared__ float os[MLA_SMALL_B][OSW];
    pdl_trigger();
    const int h = blockIdx.x, z = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int j0 = 16 * z + 2 * warp;
    const __nv_bfloat16 *W = w_uv + (size_t)h * uv_head_elems + (size_t)j0 * MLA_DL + 16 * lane;
    uint4 wv[2][2];
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
        for (int q = 0; q < 2; q++)
            wv[r][q] = __ldg(reinterpret_cast<const uint4 *>(W + (size_t)r * MLA_DL + 8 * q));
    pdl_wait();  // the weights above are never written by the chain; o_lat is
    for (int e = tid; e < B * MLA_DL; e += 256) {
        const __nv_bfloat16 *src = olat2 + ((size_t)(e / MLA_DL) * H + h) * 2 * MLA_DL;
        const int c = e % MLA_DL;
        os[e / MLA_DL][c + c / 16] =
            __bfloat162float(src[c]) + __bfloat162float(src[MLA_DL + c]);
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < 2; r++) {
        float wf[16];
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const uint32_t u[4] = {wv[r][q].x, wv[r][q].y, wv[r][q].z, wv[r][q].w};
#pragma unroll
            for (int x = 0; x < 4; x++) {
                wf[8 * q + 2 * x] = __uint_as_float(u[x] << 16);
                wf[8 * q + 2 * x + 1] = __uint_as_float(u[x] & 0xffff0000u);
            }
        }
        for (int b = 0; b < B; b++) {
            float v = 0.f;
#pragma unroll
            for (int x = 0; x < 16; x++) v = fmaf(os[b][17 * lane + x], wf[x], v);
#pragma unroll
            for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) io<OUT>::st(out + ((size_t)b * H + h) * MLA_DV + j0 + r, v);
        }
    }
}

// ---------------------------------------------------------------------------- merge
// One CTA per (head, sequence): combine the sequence's segments (max, sum, o_lat) by the
// flash-decoding identity and write o_lat as a bf16 hi/lo pair [B][H][hi 512 | lo 512] for
// mla_project_tc. Thread t owns latent elements 4t .. 4t+3. The segments' (max, sum) pairs
// are read in parallel (one per thread) and the partials eight at a time, so a sequence
// split over many clusters costs a few memory latencies, not one per segment.
__global__ void __launch_bounds__(128)
mla_merge(const float *__restrict__ part, const int *__restrict__ slot0,
          __nv_bfloat16 *__restrict__ olat2, int H) {
    constexpr int MS = 128;  // segments whose weights are staged at a time
    __shared__ float wsh[MS];
    __shared__ float red[2][4];
    pdl_trigger();
    pdl_wait();  // the partials come from the attention kernel
    const int h = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int s0 = slot0[b], s1 = slot0[b + 1];
    const size_t stride = (size_t)H * MLA_PART;
    const float *base = part + (size_t)h * MLA_PART;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    constexpr int FEW = 4;
    if (s1 - s0 <= FEW) {
        // a few segments (the common case): every thread reads their (max, sum) pairs and
        // partial rows at once, no shared memory
        float mv[FEW], lv[FEW];
        float4 pv[FEW];
#pragma unroll
        for (int i = 0; i < FEW; i++) {
            if (s0 + i < s1) {
                const float *sp = base + (size_t)(s0 + i) * stride;
                mv[i] = sp[MLA_DL];
                lv[i] = sp[MLA_DL + 1];
                pv[i] = reinterpret_cast<const float4 *>(sp)[tid];
            }
        }
        float M = -INFINITY;
#pragma unroll
        for (int i = 0; i < FEW; i++)
            if (s0 + i < s1) M = fmaxf(M, mv[i]);
        float L = 0.f;
#pragma unroll
        for (int i = 0; i < FEW; i++)
            if (s0 + i < s1) L += exp2f(mv[i] - M) * lv[i];
        const float invL = 1.f / L;
#pragma unroll
        for (int i = 0; i < FEW; i++) {
            if (s0 + i < s1) {
                const float w = exp2f(mv[i] - M) * invL;
                o.x += w * pv[i].x; o.y += w * pv[i].y; o.z += w * pv[i].z; o.w += w * pv[i].w;
            }
        }
    } else {
        // global max and sum over all segments, one segment per thread per round
        float M = -INFINITY;
        for (int s = s0 + tid; s < s1; s += 128) M = fmaxf(M, base[s * stride + MLA_DL]);
#pragma unroll
        for (int sh = 16; sh; sh >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, sh));
        if ((tid & 31) == 0) red[0][tid >> 5] = M;
        __syncthreads();
        M = fmaxf(fmaxf(red[0][0], red[0][1]), fmaxf(red[0][2], red[0][3]));
        float L = 0.f;
        for (int s = s0 + tid; s < s1; s += 128)
            L += exp2f(base[s * stride + MLA_DL] - M) * base[s * stride + MLA_DL + 1];
#pragma unroll
        for (int sh = 16; sh; sh >>= 1) L += __shfl_xor_sync(0xffffffffu, L, sh);
        if ((tid & 31) == 0) red[1][tid >> 5] = L;
        __syncthreads();
        const float invL = 1.f / ((red[1][0] + red[1][1]) + (red[1][2] + red[1][3]));
        for (int c0 = s0; c0 < s1; c0 += MS) {
            const int nc = min(MS, s1 - c0);
            if (tid < nc) wsh[tid] = exp2f(base[(c0 + tid) * stride + MLA_DL] - M) * invL;
            __syncthreads();
            int s = 0;
            for (; s + 8 <= nc; s += 8) {
                float4 p[8];
#pragma unroll
                for (int u = 0; u < 8; u++)
                    p[u] = reinterpret_cast<const float4 *>(base + (c0 + s + u) * stride)[tid];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const float w = wsh[s + u];
                    o.x += w * p[u].x; o.y += w * p[u].y; o.z += w * p[u].z; o.w += w * p[u].w;
                }
            }
            for (; s < nc; s++) {
                const float w = wsh[s];
                const float4 p = reinterpret_cast<const float4 *>(base + (c0 + s) * stride)[tid];
                o.x += w * p.x; o.y += w * p.y; o.z += w * p.z; o.w += w * p.w;
            }
            __syncthreads();  // wsh is rewritten by the next round
        }
    }
    const float ov[4] = {o.x, o.y, o.z, o.w};
    uint32_t hi[2], lo[2];
#pragma unroll
    for (int i = 0; i < 2; i++) {
        const __nv_bfloat162 t = __floats2bfloat162_rn(ov[2 * i], ov[2 * i + 1]);
        const float2 tf = __bfloat1622float2(t);
        const __nv_bfloat162 r = __floats2bfloat162_rn(ov[2 * i] - tf.x, ov[2 * i + 1] - tf.y);
        hi[i] = *reinterpret_cast<const uint32_t *>(&t);
        lo[i] = *reinterpret_cast<const uint32_t *>(&r);
    }
    __nv_bfloat16 *dst = olat2 + ((size_t)b * H + h) * 2 * MLA_DL;
    reinterpret_cast<uint2 *>(dst)[tid] = make_uint2(hi[0], hi[1]);
    reinterpret_cast<uint2 *>(dst + MLA_DL)[tid] = make_uint2(lo[0], lo[1]);
}

// ---------------------------------------------------------------------- host side
static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct MlaPlan {
    std::vector<MlaSeg> segs;
    std::vector<int> cl_begin, slot0;
    int ncl = 0;
};

static void mla_plan(const int *ctx_lens, int B, int max_clusters, MlaPlan &p) {
    std::vector<long long> nt_b((size_t)B), cstart((size_t)B + 1, 0);
    long long nt = 0;
    for (int b = 0; b < B; b++) {
        nt_b[b] = (ctx_lens[b] + MLA_TILE - 1) / MLA_TILE;
        nt += nt_b[b];
        // a sequence costs its tiles plus the fixed work of a segment
        cstart[b + 1] = cstart[b] + (nt_b[b] ? nt_b[b] + MLA_SEG_COST : 0);
    }
    // at least MLA_MIN_TILES tiles per cluster: a cluster's fixed cost (TMEM, barriers, the
    // query load) and the merge of its partial outweigh a single tile
    p.ncl = (int)std::max<long long>(
        1, std::min<long long>(max_clusters, (nt + MLA_MIN_TILES - 1) / MLA_MIN_TILES));
    p.cl_begin.assign((size_t)p.ncl + 1, 0);
    p.slot0.assign((size_t)B + 1, 0);
    // Clusters take equal shares of the cost line, on which sequence b's tile k sits at
    // cstart[b] + MLA_SEG_COST + k: a cluster given many short sequences (the early queries
    // of a causal prefill) gets fewer tiles than one given a few long ones.
    auto build = [&](bool weighted) {
        p.segs.clear();
        const long long total = weighted ? cstart[B] : nt;
        int b = 0;
        long long tb = 0;  // first tile index of sequence b on the unweighted line
        for (int c = 0; c < p.ncl; c++) {
            const long long c0 = total * c / p.ncl, c1 = total * (c + 1) / p.ncl;
            p.cl_begin[c] = (int)p.segs.size();
            while (b < B) {
                const long long pos0 = weighted ? cstart[b] + MLA_SEG_COST : tb;  // tile 0
                const long long lo = std::max(0LL, c0 - pos0), hi = std::min(nt_b[b], c1 - pos0);
                if (lo < hi) p.segs.push_back(MlaSeg{b, (int)lo, (int)hi, 0});
                if (pos0 + nt_b[b] > c1) break;  // the sequence continues in the next cluster
                tb += nt_b[b];
                b++;
            }
            if ((int)p.segs.size() == p.cl_begin[c]) return false;  // an empty cluster
        }
        p.cl_begin[p.ncl] = (int)p.segs.size();
        return true;
    };
    if (!build(true)) build(false);
    // segments come in (sequence, tile) order, so each sequence's slots are contiguous
    std::vector<int> cnt((size_t)B, 0);
    for (auto &sg : p.segs) cnt[sg.b]++;
    for (int i = 0; i < B; i++) p.slot0[i + 1] = p.slot0[i] + cnt[i];
    std::vector<int> used((size_t)B, 0);
    for (auto &sg : p.segs) sg.slot = p.slot0[sg.b] + used[sg.b]++;
}

static size_t mla_ws_bytes(const MlaPlan &p, int B, int H) {
    return align256(p.segs.size() * sizeof(MlaSeg)) + align256(p.cl_begin.size() * sizeof(int)) +
           align256(((size_t)B + 1) * sizeof(int)) + 2 * align256((size_t)B * sizeof(int)) +
           align256((size_t)B * MLA_HP * MLA_QW * 2) +
           align256(p.segs.size() * (size_t)H * MLA_PART * sizeof(float)) +
           align256((size_t)B * H * 2 * MLA_DL * 2);
}

constexpr int MLA_MAX_CLUSTERS = 74;  // 148 SMs of a B200, two per cluster

// Workspace for B queries whatever cluster count the run plans with (it uses
// min(MLA_MAX_CLUSTERS, SMs / 2)): clusters take contiguous ranges of the (query, tile) line,
// so each cluster boundary splits at most one query and a plan has at most
// B + clusters - 1 segments; mla_ws_bytes grows with the segment and cluster counts only.
static size_t mla_ws_bound(int B, int H) {
    MlaPlan p;
    p.segs.resize((size_t)B + MLA_MAX_CLUSTERS - 1);
    p.cl_begin.resize((size_t)MLA_MAX_CLUSTERS + 1);
    return mla_ws_bytes(p, B, H);
}

}  // namespace k3

using namespace k3;

extern "C" int k3cuda_mla_decode_workspace(const int *ctx_lens, int B, int H, int dl, int dv,
                                           size_t *bytes) {
    K3_ARG_CHECK(bytes && ctx_lens && B >= 0 && H >= 1 && H <= MLA_HP, "bad MLA workspace query");
    if (dl != MLA_DL || dv != MLA_DV)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "mla_decode: dl=%d dv=%d not built", dl, dv);
    for (int b = 0; b < B; b++)
        K3_ARG_CHECK(ctx_lens[b] >= 1, "ctx_lens[%d]=%d must be >= 1", b, ctx_lens[b]);
    *bytes = mla_ws_bound(B, H);
    return K3CUDA_OK;
}

extern "C" int k3cuda_mla_plan_stats(const int *ctx_lens, int B, int max_clusters, int *segments,
                                     int *clusters, size_t *bytes) {
    K3_ARG_CHECK(ctx_lens && B >= 1 && max_clusters >= 1 && segments && clusters && bytes,
                 "bad MLA plan query");
    for (int b = 0; b < B; b++)
        K3_ARG_CHECK(ctx_lens[b] >= 1, "ctx_lens[%d]=%d must be >= 1", b, ctx_lens[b]);
    MlaPlan p;
    mla_plan(ctx_lens, B, std::min(MLA_MAX_CLUSTERS, max_clusters), p);
    *segments = (int)p.segs.size();
    *clusters = p.ncl;
    *bytes = mla_ws_bytes(p, B, MLA_HP);
    return K3CUDA_OK;
}

// Every query b attends positions [0, ctx_lens[b]) of cache sequence cache_seq[b] (NULL:
// b itself) of an [n_cache][cap] latent / rope cache.
static int mla_run(k3cuda_ctx *ctx, void *out, int out_dtype, const void *q_nope,
                   const void *q_rope, const void *latent, const void *rope, const void *w_uk,
                   const void *w_uv, int uk_head_rows, int uv_head_rows,
                   const int *cache_seq, const int *ctx_lens, int B,
                   int n_cache, int cap, int H, int dn, int dr, int dl, int dv, float scale,
                   void *workspace, size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (dn != MLA_DN || dr != MLA_DR || dl != MLA_DL || dv != MLA_DV)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "mla_decode: dn=%d dr=%d dl=%d dv=%d not built",
                         dn, dr, dl, dv);
    K3_ARG_CHECK(out_dtype == K3CUDA_F32 || out_dtype == K3CUDA_BF16, "bad out_dtype");
    K3_ARG_CHECK(H >= 1 && H <= MLA_HP && B >= 0 && cap >= 1 && n_cache >= 1,
                 "bad H=%d B=%d cap=%d n_cache=%d", H, B, cap, n_cache);
    if (B == 0) return K3CUDA_OK;
    K3_ARG_CHECK(ctx_lens, "null ctx_lens");
    std::vector<int> row0((size_t)B);
    for (int b = 0; b < B; b++) {
        K3_ARG_CHECK(ctx_lens[b] >= 1 && ctx_lens[b] <= cap, "ctx_lens[%d]=%d outside [1, %d]", b,
                     ctx_lens[b], cap);
        const int cs = cache_seq ? cache_seq[b] : b;
        K3_ARG_CHECK(cs >= 0 && cs < n_cache, "cache_seq[%d]=%d outside [0, %d)", b, cs, n_cache);
        row0[(size_t)b] = cs * cap;
    }
    K3_ARG_CHECK(out && q_nope && q_rope && latent && rope && w_uk && w_uv, "null pointer");
    K3_ARG_CHECK(aligned(latent, 16) && aligned(rope, 16), "caches must be 16-byte aligned");
    K3_ARG_CHECK((long long)n_cache * cap < (1ll << 31) && (long long)B * MLA_HP < (1ll << 31),
                 "cache too large for 32-bit TMA row coordinates");
    MlaPlan p;
    mla_plan(ctx_lens, B, std::min(MLA_MAX_CLUSTERS, std::max(1, ctx->sm_count / 2)), p);
    const size_t need = mla_ws_bytes(p, B, H);
    if (workspace_bytes < need || !workspace)
        return set_error(K3CUDA_ERR_WORKSPACE, "mla_decode: workspace %zu < %zu", workspace_bytes,
                         need);
    K3_ARG_CHECK(aligned(workspace, 256), "workspace must be 256-byte aligned");
    const int nseg = (int)p.segs.size();
    char *w = (char *)workspace;
    MlaSeg *d_segs = (MlaSeg *)w;
    w += align256((size_t)nseg * sizeof(MlaSeg));
    int *d_cl = (int *)w;
    w += align256(p.cl_begin.size() * sizeof(int));
    int *d_slot0 = (int *)w;
    w += align256(((size_t)B + 1) * sizeof(int));
    int *d_lens = (int *)w;
    w += align256((size_t)B * sizeof(int));
    int *d_row0 = (int *)w;
    w += align256((size_t)B * sizeof(int));
    __nv_bfloat16 *qlat = (__nv_bfloat16 *)w;
    w += align256((size_t)B * MLA_HP * MLA_QW * 2);
    float *part = (float *)w;
    w += align256((size_t)nseg * H * MLA_PART * sizeof(float));
    __nv_bfloat16 *olat2 = (__nv_bfloat16 *)w;
    {
        // the five tables sit back to back at the start of the workspace: one image, one copy
        const size_t tbytes = (size_t)((char *)qlat - (char *)workspace);
        std::vector<unsigned char> img(tbytes, 0);
        auto put = [&](const void *dptr, const void *src, size_t n) {
            memcpy(img.data() + ((const char *)dptr - (const char *)workspace), src, n);
        };
        put(d_segs, p.segs.data(), (size_t)nseg * sizeof(MlaSeg));
        put(d_cl, p.cl_begin.data(), p.cl_begin.size() * sizeof(int));
        put(d_slot0, p.slot0.data(), ((size_t)B + 1) * sizeof(int));
        put(d_lens, ctx_lens, (size_t)B * sizeof(int));
        put(d_row0, row0.data(), (size_t)B * sizeof(int));
        if ((rc = stage_h2d(ctx, workspace, img.data(), tbytes))) return rc;
    }
    const bool small = B <= MLA_SMALL_B;  // the small absorb kernel zeroes the padded rows
    if (H < MLA_HP && !small)  // the padded query rows must score zero
        K3_CUDA_TRY(cudaMemset2DAsync(qlat + (size_t)H * MLA_QW, (size_t)MLA_HP * MLA_QW * 2, 0,
                                      (size_t)(MLA_HP - H) * MLA_QW * 2, (size_t)B, ctx->stream));

    const CUtensorMapDataType BF = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    HeadGemmMaps qmaps, pmaps;
    MlaMaps maps;
    rc = make_tmap_3d(&qmaps.a, q_nope, BF, 2, MLA_DN, H, B, MLA_DN * 2, (uint64_t)H * MLA_DN * 2,
                      64, 1, 128);
    if (!rc)
        rc = make_tmap_3d(&qmaps.b, w_uk, BF, 2, MLA_DL, MLA_DN, H, MLA_DL * 2,
                          (uint64_t)uk_head_rows * MLA_DL * 2, 64, 64, 1);
    if (!rc)
        rc = make_tmap_2d(&maps.lat, latent, BF, 2, MLA_DL, (uint64_t)n_cache * cap, MLA_DL * 2,
                          64, MLA_TILE);
    if (!rc)
        rc = make_tmap_2d(&maps.rope, rope, BF, 2, MLA_DR, (uint64_t)n_cache * cap, MLA_DR * 2,
                          64, MLA_TILE);
    if (!rc)
        rc = make_tmap_3d(&pmaps.a, olat2, BF, 2, 2 * MLA_DL, H, B, 2 * MLA_DL * 2,
                          (uint64_t)H * 2 * MLA_DL * 2, 64, 1, 128);
    if (!rc)
        rc = make_tmap_3d(&pmaps.b, w_uv, BF, 2, MLA_DL, MLA_DV, H, MLA_DL * 2,
                          (uint64_t)uv_head_rows * MLA_DL * 2, 64, 128, 1);
    if (rc) return rc;
    K3_ARG_CHECK(aligned(q_nope, 16) && aligned(q_rope, 16) && aligned(w_uk, 16) &&
                     aligned(w_uv, 16),
                 "MLA inputs must be 16-byte aligned");

    const dim3 hgrid(H, (B + 127) / 128);
    if (small) {
        const dim3 g(MLA_HP, MLA_DL / 128);
        const __nv_bfloat16 *qn = (const __nv_bfloat16 *)q_nope, *qr = (const __nv_bfloat16 *)q_rope,
                            *wk = (const __nv_bfloat16 *)w_uk;
        const long long uk = (long long)uk_head_rows * MLA_DL;
        const char *nm = "mla_q_absorb_small";
        const dim3 blk(256);
        if (B <= 1)
            rc = launch_pdl(ctx, ctx->stream, nm, mla_q_absorb_small<1>, g, blk, 0, qn, qr, wk, uk,
                            qlat, B, H);
        else if (B <= 2)
            rc = launch_pdl(ctx, ctx->stream, nm, mla_q_absorb_small<2>, g, blk, 0, qn, qr, wk, uk,
                            qlat, B, H);
        else if (B <= 4)
            rc = launch_pdl(ctx, ctx->stream, nm, mla_q_absorb_small<4>, g, blk, 0, qn, qr, wk, uk,
                            qlat, B, H);
        else
            rc = launch_pdl(ctx, ctx->stream, nm, mla_q_absorb_small<8>, g, blk, 0, qn, qr, wk, uk,
                            qlat, B, H);
    } else {
        const int qsmem = 2 * 16384 + 8 * 8192 + 1024;
        if (int rc_ = set_smem(mla_q_absorb_tc, qsmem)) return rc_;
        const dim3 qgrid(H, (B + 127) / 128, 2);  // two 256-column halves of q_lat per head
        mla_q_absorb_tc<<<qgrid, 128, qsmem, ctx->stream>>>(qmaps, (const __nv_bfloat16 *)q_rope,
                                                            qlat, B, H, ctx->err_word);
        rc = after_launch(ctx, "mla_q_absorb_tc");
    }
    if (rc) return rc;

    if (int rc_ = set_smem(mla_attend_tc, MLA_SMEM)) return rc_;
    const float scale_log2e = scale * 1.4426950408889634f;
    rc = launch_pdl(ctx, ctx->stream, "mla_attend_tc", mla_attend_tc, dim3(2 * p.ncl),
                    dim3(MLA_THREADS), MLA_SMEM, maps, (const MlaSeg *)d_segs, (const int *)d_cl,
                    (const int *)d_lens, (const __nv_bfloat16 *)qlat, part, H, (const int *)d_row0,
                    scale_log2e, ctx->err_word);
    if (rc) return rc;

    rc = launch_pdl(ctx, ctx->stream, "mla_merge", mla_merge, dim3(H, B), dim3(128), 0,
                    (const float *)part, (const int *)d_slot0, olat2, H);
    if (rc) return rc;

    if (small) {
        const dim3 pgrid(H, MLA_DV / 16);
        const long long uv = (long long)uv_head_rows * MLA_DL;
        const __nv_bfloat16 *o2 = olat2, *wu = (const __nv_bfloat16 *)w_uv;
        if (out_dtype == K3CUDA_BF16)
            return launch_pdl(ctx, ctx->stream, "mla_project_small",
                              mla_project_small<__nv_bfloat16>, pgrid, dim3(256), 0, o2, wu, uv,
                              (__nv_bfloat16 *)out, B, H);
        return launch_pdl(ctx, ctx->stream, "mla_project_small", mla_project_small<float>, pgrid,
                          dim3(256), 0, o2, wu, uv, (float *)out, B, H);
    }
    const int psmem = 3 * 2 * 16384 + 1024;
    if (out_dtype == K3CUDA_BF16) {
        if (int rc_ = set_smem(mla_project_tc<__nv_bfloat16>, psmem)) return rc_;
        mla_project_tc<__nv_bfloat16><<<hgrid, 128, psmem, ctx->stream>>>(
            pmaps, (__nv_bfloat16 *)out, B, H, ctx->err_word);
    } else {
        if (int rc_ = set_smem(mla_project_tc<float>, psmem)) return rc_;
        mla_project_tc<float><<<hgrid, 128, psmem, ctx->stream>>>(pmaps, (float *)out, B, H,
                                                                  ctx->err_word);
    }
    return after_launch(ctx, "mla_project_tc");
}

namespace k3 {
// The causal attention of one prefill chunk / decode token of one sequence for the MLA layer:
// queries b = 0..T-1 at positions cached + b over the sequence's cache, with W_UK and W_UV
// read in place from kv_b [H][256][512] bf16 (per head 128 W_UK rows, then 128 W_UV rows).
int mla_attend_kvb(k3cuda_ctx *ctx, float *acc, const void *q_nope, const void *q_rope,
                   const void *latent, const void *rope, const void *kv_b, int T, int cached,
                   int cap, int H, float scale, void *workspace, size_t workspace_bytes) {
    std::vector<int> seq((size_t)T, 0), lens((size_t)T);
    for (int t = 0; t < T; t++) lens[(size_t)t] = cached + t + 1;
    const char *kb = (const char *)kv_b;
    return mla_run(ctx, acc, K3CUDA_F32, q_nope, q_rope, latent, rope, kb,
                   kb + (size_t)MLA_DN * MLA_DL * 2, MLA_DN + MLA_DV, MLA_DN + MLA_DV,
                   seq.data(), lens.data(), T, 1, cap, H, MLA_DN, MLA_DR, MLA_DL, MLA_DV, scale,
                   workspace, workspace_bytes);
}

size_t mla_attend_kvb_workspace(int T, int cached, int H) {
    (void)cached;
    return mla_ws_bound(T, H);
}
}  // namespace k3

extern "C" int k3cuda_mla_decode(k3cuda_ctx *ctx, void *out, int out_dtype, const void *q_nope,
                                 const void *q_rope, const void *latent, const void *rope,
                                 const void *w_uk, const void *w_uv, const int *ctx_lens, int B,
                                 int cap, int H, int dn, int dr, int dl, int dv, float scale,
                                 void *workspace, size_t workspace_bytes) {
    return mla_run(ctx, out, out_dtype, q_nope, q_rope, latent, rope, w_uk, w_uv, MLA_DN, MLA_DV,
                   nullptr, ctx_lens, B, B, cap, H, dn, dr, dl, dv, scale, workspace,
                   workspace_bytes);
}

extern "C" int k3cuda_mla_attend(k3cuda_ctx *ctx, void *out, int out_dtype, const void *q_nope,
                                 const void *q_rope, const void *latent, const void *rope,
                                 const void *w_uk, const void *w_uv, const int *cache_seq,
                                 const int *ctx_lens, int B, int n_cache, int cap, int H, int dn,
                                 int dr, int dl, int dv, float scale, void *workspace,
                                 size_t workspace_bytes) {
    K3_ARG_CHECK(cache_seq || B == 0, "mla_attend: null cache_seq");
    return mla_run(ctx, out, out_dtype, q_nope, q_rope, latent, rope, w_uk, w_uv, MLA_DN, MLA_DV,
                   cache_seq, ctx_lens, B, n_cache, cap, H, dn, dr, dl, dv, scale, workspace,
                   workspace_bytes);
}

// ------------------------------------------------------------------- cache append
// One row per token: latent[seq][pos0 + t] = bf16(kv_a_norm(ct[t][0:512])) and
// rope[seq][pos0 + t] = bf16(ct[t][512:576]) (k3_ops.c:363-366: the norm covers the latent
// only). The sum of squares is taken in double and the scale formed in double, as
// k3_rmsnorm does (k3_ops.c:94-101), so the normalised fp32 values match the reference's
// before the bf16 rounding. 128 threads, 4 latent values and half a rope value each.
__global__ void __launch_bounds__(128) mla_cache_append_k(
    __nv_bfloat16 *__restrict__ latent, __nv_bfloat16 *__restrict__ rope,
    const float *__restrict__ ct, const float *__restrict__ w, float eps, long long row_base) {
    pdl_trigger();
    pdl_wait();
    __shared__ double red[4];
    const int t = blockIdx.x, tid = threadIdx.x;
    const float *src = ct + (size_t)t * MLA_QW;
    const float4 x = reinterpret_cast<const float4 *>(src)[tid];
    double ss = (double)x.x * x.x + (double)x.y * x.y + (double)x.z * x.z + (double)x.w * x.w;
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    ss = (red[0] + red[1]) + (red[2] + red[3]);
    const float inv = (float)(1.0 / sqrt(ss / (double)MLA_DL + (double)eps));
    const float4 g = reinterpret_cast<const float4 *>(w)[tid];
    const size_t row = (size_t)(row_base + t);
    __nv_bfloat16 *dl = latent + row * MLA_DL + 4 * tid;
    const __nv_bfloat162 a = __floats2bfloat162_rn(g.x * x.x * inv, g.y * x.y * inv);
    const __nv_bfloat162 b = __floats2bfloat162_rn(g.z * x.z * inv, g.w * x.w * inv);
    reinterpret_cast<__nv_bfloat162 *>(dl)[0] = a;
    reinterpret_cast<__nv_bfloat162 *>(dl)[1] = b;
    if (tid < MLA_DR / 2) {
        const float2 r = reinterpret_cast<const float2 *>(src + MLA_DL)[tid];
        reinterpret_cast<__nv_bfloat162 *>(rope + row * MLA_DR)[tid] = __floats2bfloat162_rn(r.x, r.y);
    }
}

extern "C" int k3cuda_mla_cache_append(k3cuda_ctx *ctx, void *latent, void *rope,
                                       const float *ct, const float *kv_a_norm, float eps,
                                       int seq, int pos0, int T, int n_cache, int cap, int dl,
                                       int dr) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (dl != MLA_DL || dr != MLA_DR)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "mla_cache_append: dl=%d dr=%d not built", dl, dr);
    K3_ARG_CHECK(T >= 0 && seq >= 0 && seq < n_cache && pos0 >= 0 && (long long)pos0 + T <= cap,
                 "mla_cache_append: seq=%d pos0=%d T=%d outside [%d][%d]", seq, pos0, T, n_cache,
                 cap);
    if (T == 0) return K3CUDA_OK;
    K3_ARG_CHECK(latent && rope && ct && kv_a_norm, "mla_cache_append: null pointer");
    K3_ARG_CHECK(aligned(latent, 16) && aligned(rope, 16) && aligned(ct, 16) &&
                     aligned(kv_a_norm, 16),
                 "mla_cache_append: pointers must be 16-byte aligned");
    return launch_pdl(ctx, ctx->stream, "mla_cache_append", mla_cache_append_k, dim3(T),
                      dim3(128), 0, (__nv_bfloat16 *)latent, (__nv_bfloat16 *)rope, ct, kv_a_norm,
                      eps, (long long)seq * cap + pos0);
}
