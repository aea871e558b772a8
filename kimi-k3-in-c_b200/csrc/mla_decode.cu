// mla_decode.cu -- absorbed MLA decode over the compressed latent cache, on tcgen05.
//
// Replaces the per-head attention loop of k3_mla_cached (reference src/core/k3_ops.c:
// 381-411) for one query token per sequence. The reference caches the EXPANDED keys and
// values (k3_ops.c:304-315, 351-367); here the cache holds the latent c_s (512 wide) and the
// shared rope slot r_s (64), and the per-head blocks of kv_b are folded into the query and
// the output:
//     q_lat = W_UK^T q_nope                       mla_q_absorb      (bf16 [B][128][576])
//     S     = [q_lat | q_rope] . [c_s | r_s]^T    mla_attend_tc     (tcgen05, fp32 in TMEM)
//     P     = softmax(S * scale)                  mla_attend_tc     (fp32 on CUDA cores)
//     o_lat = P . C                               mla_attend_tc     (tcgen05, fp32 in TMEM)
//     out   = W_UV o_lat                          mla_merge_project (split-K merge + GEMM)
//
// mla_attend_tc runs as clusters of two CTAs (one SM each). All 128 heads are the MMA's M.
// The 576-wide contraction of S is split across the pair -- rank 0 takes latent dims
// [0,256) and the 64 rope dims, rank 1 latent dims [256,512) -- and each rank accumulates
// the output for its own 256 latent dims, which are exactly the dims whose tiles it already
// holds. Per 64-token tile each rank computes its partial S, the ranks exchange the partials
// through distributed shared memory, both add them in the same order (rank 0's + rank 1's),
// so both derive the same softmax, and each multiplies P by its half of the tile. Per SM:
//   shared  Q half 80 KB + 2 KV stages x 40 KB + P 16 KB + exchange 32 KB   (~209 KB)
//   TMEM    S double buffer 2 x 64 columns + O 256 columns                   (of 512)
// Warp roles: warp 0 issues TMA loads, warp 1 allocates TMEM and issues the MMAs, warps 2-5
// (one thread per head = TMEM lane) run the exchange, the softmax and the epilogue. The
// running max is only moved when it grows by more than 2^8 (a lazy rescale: numerator and
// denominator use the same stale max, so the result is exact), which keeps the O rescale in
// TMEM off the common path.
//
// Work: the (sequence, 64-token tile) list is cut into equal contiguous ranges, one per
// cluster; a range that crosses sequences becomes several segments, each writing a partial
// (max, sum, o_lat) per head; mla_merge_project combines the segments of every sequence
// (the flash-decoding identity) and applies W_UV.
//
// Every wait is bounded (sm100.cuh): on a timeout the kernel records an error word, skips
// the rest of its work, waits briefly for its own loads and frees TMEM; k3cuda_sync then
// reports K3CUDA_ERR_TIMEOUT.
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
constexpr int MLA_NST = 2;                 // KV pipeline stages
constexpr int MLA_QBLK = MLA_HP * 128;     // bytes of one 64-dim block of Q (128 rows x 128 B)
constexpr int MLA_KVBLK = MLA_TILE * 128;  // bytes of one 64-dim block of a KV tile
constexpr int MLA_NBLK = 5;                // dim blocks of rank 0 (4 latent + rope); rank 1: 4
constexpr int MLA_OFF_Q = 0;
constexpr int MLA_OFF_KV = MLA_OFF_Q + MLA_NBLK * MLA_QBLK;
constexpr int MLA_OFF_P = MLA_OFF_KV + MLA_NST * MLA_NBLK * MLA_KVBLK;
constexpr int MLA_OFF_X = MLA_OFF_P + MLA_HP * 128;
constexpr int MLA_SMEM = MLA_OFF_X + MLA_HP * MLA_TILE * 4 + 1024;  // + alignment slack
constexpr int MLA_PART = MLA_DL + 4;       // floats per (segment, head): o_lat, max, sum, pad
                                           // (rows stay 16-byte aligned for float4 stores)
constexpr int MLA_TM_S = 0, MLA_TM_O = 128, MLA_TM_COLS = 512;
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

// ------------------------------------------------------------------------- q absorb
// qlat[b][h][0:512] = W_UK[h]^T q_nope[b][h], qlat[b][h][512:576] = q_rope[b][h], bf16, with
// rows h >= H zero. One CTA per (padded head, group of 16 sequences); thread l owns latent
// columns l and l + 256.
__global__ void __launch_bounds__(256)
mla_q_absorb(const __nv_bfloat16 *__restrict__ q_nope, const __nv_bfloat16 *__restrict__ q_rope,
             const __nv_bfloat16 *__restrict__ w_uk, __nv_bfloat16 *__restrict__ qlat, int B,
             int H) {
    __shared__ float sq[16][MLA_DN];
    const int h = blockIdx.x, b0 = blockIdx.y * 16, tid = threadIdx.x;
    const bool live = h < H;
    for (int e = tid; e < 16 * MLA_DN; e += 256) {
        const int bb = e / MLA_DN, i = e % MLA_DN;
        sq[bb][i] = (live && b0 + bb < B) ? bf(q_nope + ((size_t)(b0 + bb) * H + h) * MLA_DN + i)
                                          : 0.f;
    }
    __syncthreads();
    float acc0[16], acc1[16];
#pragma unroll
    for (int bb = 0; bb < 16; bb++) acc0[bb] = acc1[bb] = 0.f;
    if (live) {
        const __nv_bfloat16 *W = w_uk + (size_t)h * MLA_DN * MLA_DL;
        for (int i = 0; i < MLA_DN; i++) {
            const float w0 = bf(W + (size_t)i * MLA_DL + tid);
            const float w1 = bf(W + (size_t)i * MLA_DL + tid + 256);
#pragma unroll
            for (int bb = 0; bb < 16; bb++) {
                acc0[bb] += sq[bb][i] * w0;
                acc1[bb] += sq[bb][i] * w1;
            }
        }
    }
#pragma unroll
    for (int bb = 0; bb < 16; bb++) {
        if (b0 + bb < B) {
            __nv_bfloat16 *dst = qlat + ((size_t)(b0 + bb) * MLA_HP + h) * MLA_QW;
            dst[tid] = __float2bfloat16_rn(acc0[bb]);
            dst[tid + 256] = __float2bfloat16_rn(acc1[bb]);
            if (tid < MLA_DR)
                dst[MLA_DL + tid] = live ? q_rope[((size_t)(b0 + bb) * H + h) * MLA_DR + tid]
                                         : __float2bfloat16_rn(0.f);
        }
    }
}

// ---------------------------------------------------------------------------- attend
struct MlaSeg {
    int b, t0, t1, slot;  // sequence, tile range [t0, t1), partial slot
};

struct MlaMaps {
    CUtensorMap q, lat, rope;
};

struct MlaBars {
    uint64_t kv_full[MLA_NST], kv_empty[MLA_NST];
    uint64_t q_full, q_empty;
    uint64_t s_full[2], s_empty[2];
    uint64_t p_full, pv_done;
    uint64_t x_full, x_empty;
    uint32_t tmem_base;
};

__global__ void __launch_bounds__(192, 1) __cluster_dims__(2, 1, 1)
mla_attend_tc(const __grid_constant__ MlaMaps maps, const MlaSeg *__restrict__ segs,
              const int *__restrict__ cl_begin, const int *__restrict__ ctx_lens,
              float *__restrict__ part, int H, int cap, float scale_log2e,
              unsigned *__restrict__ err) {
    extern __shared__ uint8_t smraw[];
    uint8_t *sm = (uint8_t *)(((uintptr_t)smraw + 1023) & ~(uintptr_t)1023);
    __shared__ MlaBars bars;
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
        mbar_init(&bars.q_full, 1);
        mbar_init(&bars.q_empty, 1);
        for (int s = 0; s < 2; s++) {
            mbar_init(&bars.s_full[s], 1);
            mbar_init(&bars.s_empty[s], 128);
        }
        mbar_init(&bars.p_full, 128);
        mbar_init(&bars.pv_done, 1);
        mbar_init(&bars.x_full, 128);
        mbar_init(&bars.x_empty, 128);
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
            prefetch_tmap(&maps.q);
            prefetch_tmap(&maps.lat);
            prefetch_tmap(&maps.rope);
            int g = 0, nq = 0, prev_b = -1;
            int last_use[MLA_NST] = {-1, -1};
            bool ok = true;
            for (int si = sbeg; si < send && ok; si++) {
                const MlaSeg sg = segs[si];
                if (sg.b != prev_b) {
                    if (nq > 0) ok = mbar_wait(&bars.q_empty, (nq - 1) & 1, err, 0x101);
                    if (!ok) break;
                    mbar_expect_tx(&bars.q_full, nblk * MLA_QBLK);
                    for (int kb = 0; kb < nblk; kb++) {
                        const int col = kb < 4 ? dim0 + kb * 64 : MLA_DL;
                        tma_load_2d(sm + MLA_OFF_Q + kb * MLA_QBLK, &maps.q, &bars.q_full, col,
                                    sg.b * MLA_HP);
                    }
                    nq++;
                    prev_b = sg.b;
                }
                for (int t = sg.t0; t < sg.t1; t++, g++) {
                    const int st = g % MLA_NST, n = g / MLA_NST;
                    if (n > 0 && !(ok = mbar_wait(&bars.kv_empty[st], (n - 1) & 1, err, 0x102)))
                        break;
                    mbar_expect_tx(&bars.kv_full[st], nblk * MLA_KVBLK);
                    uint8_t *dst = sm + MLA_OFF_KV + st * MLA_NBLK * MLA_KVBLK;
                    const int row = sg.b * cap + t * MLA_TILE;
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
        // ----------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_f16(128, MLA_TILE, false, false);
            constexpr uint32_t id_o = idesc_f16(128, 256, false, true);
            int g = 0, nq = 0, prev_b = -1;
            bool ok = true;
            int pend = -1;  // tile whose PV is still to be issued
            bool pend_first = false;
            auto issue_pv = [&](int gp, bool first) -> bool {
                if (!mbar_wait(&bars.p_full, gp & 1, err, 0x203)) return false;
                tc_fence_after();
                const uint8_t *kv = sm + MLA_OFF_KV + (gp % MLA_NST) * MLA_NBLK * MLA_KVBLK;
                const uint8_t *P = sm + MLA_OFF_P;
#pragma unroll
                for (int ks = 0; ks < MLA_TILE / 16; ks++) {
                    const uint64_t ad = sdesc_kmajor(smem_u32(P + ks * 32));
                    const uint64_t bd = sdesc_mnmajor(smem_u32(kv + ks * 2048), MLA_KVBLK);
                    mma_bf16_ss(tbase + MLA_TM_O, ad, bd, id_o, (first && ks == 0) ? 0u : 1u);
                }
                mma_commit(&bars.kv_empty[gp % MLA_NST]);
                mma_commit(&bars.pv_done);
                return true;
            };
            for (int si = sbeg; si < send && ok; si++) {
                const MlaSeg sg = segs[si];
                const bool qlast = si + 1 >= send || segs[si + 1].b != sg.b;
                if (sg.b != prev_b) {
                    if (!(ok = mbar_wait(&bars.q_full, nq & 1, err, 0x201))) break;
                    nq++;
                    prev_b = sg.b;
                }
                for (int t = sg.t0; t < sg.t1 && ok; t++, g++) {
                    const int st = g % MLA_NST, sb = g & 1;
                    if (!(ok = mbar_wait(&bars.kv_full[st], (g / MLA_NST) & 1, err, 0x202))) break;
                    if (g >= 2 &&
                        !(ok = mbar_wait(&bars.s_empty[sb], ((g >> 1) - 1) & 1, err, 0x204)))
                        break;
                    tc_fence_after();
                    const uint8_t *kv = sm + MLA_OFF_KV + st * MLA_NBLK * MLA_KVBLK;
                    for (int kb = 0; kb < nblk; kb++)
#pragma unroll
                        for (int ks = 0; ks < 4; ks++) {
                            const uint64_t ad =
                                sdesc_kmajor(smem_u32(sm + MLA_OFF_Q + kb * MLA_QBLK + ks * 32));
                            const uint64_t bd =
                                sdesc_kmajor(smem_u32(kv + kb * MLA_KVBLK + ks * 32));
                            mma_bf16_ss(tbase + MLA_TM_S + sb * MLA_TILE, ad, bd, id_s,
                                        (kb | ks) ? 1u : 0u);
                        }
                    mma_commit(&bars.s_full[sb]);
                    if (qlast && t + 1 == sg.t1) mma_commit(&bars.q_empty);
                    if (pend >= 0 && !(ok = issue_pv(pend, pend_first))) break;
                    pend = g;
                    pend_first = t == sg.t0;
                }
            }
            if (ok && pend >= 0) issue_pv(pend, pend_first);
        }
    } else {
        // -------------------------------------------- exchange, softmax, epilogue
        const int row = 32 * (warp & 3) + lane;  // head == TMEM lane
        const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
        const float4 *X4 = reinterpret_cast<const float4 *>(sm + MLA_OFF_X);
        const uint32_t xpeer = map_peer(smem_u32(sm + MLA_OFF_X), peer);
        uint8_t *P = sm + MLA_OFF_P;
        float m_ref = -INFINITY, l = 0.f;
        int g = 0, cur_slot = -1;
        bool ok = true;
        auto epilogue = [&](int slot) {  // warp-collective: every lane loads its row
            float *dst = part + ((size_t)slot * H + row) * MLA_PART;
            for (int c = 0; c < 256; c += 16) {
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
            if (rank == 0 && row < H) {
                dst[MLA_DL] = m_ref;
                dst[MLA_DL + 1] = l;
            }
        };
        for (int si = sbeg; si < send && ok; si++) {
            const MlaSeg sg = segs[si];
            const int clen = ctx_lens[sg.b];
            for (int t = sg.t0; t < sg.t1; t++, g++) {
                const int sb = g & 1;
                float s[MLA_TILE];
                if (!(ok = warp_wait(&bars.s_full[sb], (g >> 1) & 1, err, 0x301))) break;
                tc_fence_after();
#pragma unroll
                for (int c = 0; c < MLA_TILE; c += 16) {
                    float v[16];
                    tmem_ld16(tbase + lane_off + MLA_TM_S + sb * MLA_TILE + c, v);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; i++) s[c + i] = v[i];
                }
                tc_fence_before();
                mbar_arrive(&bars.s_empty[sb]);
                // exchange partial scores with the peer; X4[i * 128 + row] = float4 i of `row`
                if (g > 0 && !(ok = warp_wait(&bars.x_empty, (g - 1) & 1, err, 0x302, true))) break;
#pragma unroll
                for (int i = 0; i < MLA_TILE / 4; i++)
                    st_cluster_v4(xpeer + (uint32_t)((i * MLA_HP + row) * 16), s[4 * i],
                                  s[4 * i + 1], s[4 * i + 2], s[4 * i + 3]);
                mbar_arrive_cluster(&bars.x_full, peer);
                if (!(ok = warp_wait(&bars.x_full, g & 1, err, 0x303, true))) break;
                const int valid = clen - t * MLA_TILE;
                float mx = -INFINITY;
#pragma unroll
                for (int i = 0; i < MLA_TILE / 4; i++) {
                    const float4 o = X4[i * MLA_HP + row];
                    const float ov[4] = {o.x, o.y, o.z, o.w};
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int c = 4 * i + j;
                        const float tot = rank == 0 ? s[c] + ov[j] : ov[j] + s[c];
                        s[c] = c < valid ? tot * scale_log2e : -INFINITY;
                        mx = fmaxf(mx, s[c]);
                    }
                }
                mbar_arrive_cluster(&bars.x_empty, peer);
                // PV of the previous tile done: P buffer free, O stable
                if (g > 0 && !(ok = warp_wait(&bars.pv_done, (g - 1) & 1, err, 0x304))) break;
                tc_fence_after();
                if (t == sg.t0) {
                    if (cur_slot >= 0) epilogue(cur_slot);
                    cur_slot = sg.slot;
                    m_ref = mx;
                    l = 0.f;
                } else {
                    const bool grow = mx > m_ref + MLA_RESCALE_LOG2;
                    if (__any_sync(0xffffffffu, grow)) {
                        const float f = grow ? exp2f(m_ref - mx) : 1.f;
                        for (int c = 0; c < 256; c += 16) {
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
                // P row (bf16, 128-byte swizzle: 16-byte chunk c of row r sits at c ^ (r & 7))
                float rs = 0.f;
                uint32_t pk[MLA_TILE / 2];
#pragma unroll
                for (int c = 0; c < MLA_TILE; c += 2) {
                    const float p0 = exp2f(s[c] - m_ref), p1 = exp2f(s[c + 1] - m_ref);
                    rs += p0 + p1;
                    const __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
                    pk[c / 2] = *reinterpret_cast<const uint32_t *>(&h2);
                }
                l += rs;
#pragma unroll
                for (int c = 0; c < 8; c++)
                    *reinterpret_cast<uint4 *>(P + row * 128 + ((c ^ (row & 7)) * 16)) =
                        make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
                if (valid < MLA_TILE) {
                    // rows past the context may hold anything (even NaN): zero this rank's
                    // value rows there so that P = 0 times them stays 0
                    uint8_t *kv = sm + MLA_OFF_KV + (g % MLA_NST) * MLA_NBLK * MLA_KVBLK;
                    const int nz = (MLA_TILE - valid) * 8;  // 16-byte chunks per block
                    for (int e = row; e < 4 * nz; e += 128) {
                        const int kb = e / nz, r = valid + (e % nz) / 8, c = e % 8;
                        *reinterpret_cast<uint4 *>(kv + kb * MLA_KVBLK + r * 128 + c * 16) =
                            make_uint4(0, 0, 0, 0);
                    }
                }
                fence_async_shared();
                tc_fence_before();
                mbar_arrive(&bars.p_full);
            }
        }
        if (ok && g > 0 && warp_wait(&bars.pv_done, (g - 1) & 1, err, 0x305)) {
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

// ------------------------------------------------------------------ merge + project
// One CTA per head: merge every sequence's segments (max, sum, o_lat) into o_lat, then
// out[b][h][:] = W_UV[h] o_lat[b] as a [64 x 512] x [512 x 128] tile product per 64
// sequences (each thread 4 sequences x 8 outputs).
template <typename OUT>
__global__ void __launch_bounds__(256)
mla_merge_project(const float *__restrict__ part, const int *__restrict__ slot0,
                  const __nv_bfloat16 *__restrict__ w_uv, OUT *__restrict__ out, int B, int H,
                  int nslots) {
    extern __shared__ float msm[];
    float *wsl = msm;             // [nslots] merge weight of each slot (this head)
    float *sA = wsl + nslots;     // [64 b][65] o_lat chunk (padded)
    float *sW = sA + 64 * 65;     // [128 j][65] W_UV chunk (padded)
    const int h = blockIdx.x, tid = threadIdx.x;
    const size_t hs = (size_t)h * MLA_PART, sstride = (size_t)H * MLA_PART;
    for (int b = tid; b < B; b += 256) {
        float M = -INFINITY;
        for (int s = slot0[b]; s < slot0[b + 1]; s++) M = fmaxf(M, part[s * sstride + hs + MLA_DL]);
        float L = 0.f;
        for (int s = slot0[b]; s < slot0[b + 1]; s++)
            L += exp2f(part[s * sstride + hs + MLA_DL] - M) * part[s * sstride + hs + MLA_DL + 1];
        for (int s = slot0[b]; s < slot0[b + 1]; s++)
            wsl[s] = exp2f(part[s * sstride + hs + MLA_DL] - M) / L;
    }
    __syncthreads();
    const int tb = tid / 16, tj = tid % 16;  // 16 x 16 threads: 4 b x 8 j each
    const __nv_bfloat16 *W = w_uv + (size_t)h * MLA_DV * MLA_DL;
    for (int b0 = 0; b0 < B; b0 += 64) {
        float acc[4][8];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 8; j++) acc[i][j] = 0.f;
        for (int k0 = 0; k0 < MLA_DL; k0 += 64) {
            __syncthreads();
            for (int e = tid; e < 64 * 64; e += 256) {
                const int bb = e / 64, kk = e % 64, b = b0 + bb;
                float a = 0.f;
                if (b < B)
                    for (int s = slot0[b]; s < slot0[b + 1]; s++)
                        a += wsl[s] * part[s * sstride + hs + k0 + kk];
                sA[bb * 65 + kk] = a;
            }
            for (int e = tid; e < 128 * 64; e += 256) {
                const int j = e / 64, kk = e % 64;
                sW[j * 65 + kk] = bf(W + (size_t)j * MLA_DL + k0 + kk);
            }
            __syncthreads();
#pragma unroll 4
            for (int kk = 0; kk < 64; kk++) {
                float a[4], w[8];
#pragma unroll
                for (int i = 0; i < 4; i++) a[i] = sA[(tb * 4 + i) * 65 + kk];
#pragma unroll
                for (int j = 0; j < 8; j++) w[j] = sW[(tj + 16 * j) * 65 + kk];
#pragma unroll
                for (int i = 0; i < 4; i++)
#pragma unroll
                    for (int j = 0; j < 8; j++) acc[i][j] += a[i] * w[j];
            }
        }
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int b = b0 + tb * 4 + i;
            if (b < B) {
#pragma unroll
                for (int j = 0; j < 8; j++)
                    io<OUT>::st(out + ((size_t)b * H + h) * MLA_DV + tj + 16 * j, acc[i][j]);
            }
        }
    }
}

// ---------------------------------------------------------------------- host side
static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

struct MlaPlan {
    std::vector<MlaSeg> segs;
    std::vector<int> cl_begin, slot0;
    int ncl = 0;
};

static void mla_plan(const int *ctx_lens, int B, int max_clusters, MlaPlan &p) {
    std::vector<long long> tstart((size_t)B + 1, 0);
    for (int b = 0; b < B; b++) tstart[b + 1] = tstart[b] + (ctx_lens[b] + MLA_TILE - 1) / MLA_TILE;
    const long long nt = tstart[B];
    p.ncl = (int)std::max<long long>(1, std::min<long long>(max_clusters, nt));
    p.segs.clear();
    p.cl_begin.assign((size_t)p.ncl + 1, 0);
    p.slot0.assign((size_t)B + 1, 0);
    int b = 0;
    for (int c = 0; c < p.ncl; c++) {
        const long long g0 = nt * c / p.ncl, g1 = nt * (c + 1) / p.ncl;
        p.cl_begin[c] = (int)p.segs.size();
        long long g = g0;
        while (g < g1) {
            while (tstart[b + 1] <= g) b++;
            const long long e = std::min(g1, tstart[b + 1]);
            p.segs.push_back(MlaSeg{b, (int)(g - tstart[b]), (int)(e - tstart[b]), 0});
            g = e;
        }
    }
    p.cl_begin[p.ncl] = (int)p.segs.size();
    // segments come in (sequence, tile) order, so each sequence's slots are contiguous
    std::vector<int> cnt((size_t)B, 0);
    for (auto &s : p.segs) cnt[s.b]++;
    for (int i = 0; i < B; i++) p.slot0[i + 1] = p.slot0[i] + cnt[i];
    std::vector<int> used((size_t)B, 0);
    for (auto &s : p.segs) s.slot = p.slot0[s.b] + used[s.b]++;
}

static size_t mla_ws_bytes(const MlaPlan &p, int B, int H) {
    return align256(p.segs.size() * sizeof(MlaSeg)) + align256(p.cl_begin.size() * sizeof(int)) +
           align256(((size_t)B + 1) * sizeof(int)) + align256((size_t)B * sizeof(int)) +
           align256((size_t)B * MLA_HP * MLA_QW * 2) +
           align256(p.segs.size() * (size_t)H * MLA_PART * sizeof(float));
}

constexpr int MLA_MAX_CLUSTERS = 74;  // 148 SMs of a B200, two per cluster

}  // namespace k3

using namespace k3;

extern "C" int k3cuda_mla_decode_workspace(const int *ctx_lens, int B, int H, int dl, int dv,
                                           size_t *bytes) {
    K3_ARG_CHECK(bytes && ctx_lens && B >= 0 && H >= 1 && H <= MLA_HP, "bad MLA workspace query");
    if (dl != MLA_DL || dv != MLA_DV)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "mla_decode: dl=%d dv=%d not built", dl, dv);
    for (int b = 0; b < B; b++)
        K3_ARG_CHECK(ctx_lens[b] >= 1, "ctx_lens[%d]=%d must be >= 1", b, ctx_lens[b]);
    MlaPlan p;
    mla_plan(ctx_lens, B, MLA_MAX_CLUSTERS, p);
    *bytes = mla_ws_bytes(p, B, H);
    return K3CUDA_OK;
}

extern "C" int k3cuda_mla_decode(k3cuda_ctx *ctx, void *out, int out_dtype, const void *q_nope,
                                 const void *q_rope, const void *latent, const void *rope,
                                 const void *w_uk, const void *w_uv, const int *ctx_lens, int B,
                                 int cap, int H, int dn, int dr, int dl, int dv, float scale,
                                 void *workspace, size_t workspace_bytes) {
    int rc = enter(ctx);
    if (rc) return rc;
    if (dn != MLA_DN || dr != MLA_DR || dl != MLA_DL || dv != MLA_DV)
        return set_error(K3CUDA_ERR_UNSUPPORTED, "mla_decode: dn=%d dr=%d dl=%d dv=%d not built",
                         dn, dr, dl, dv);
    K3_ARG_CHECK(out_dtype == K3CUDA_F32 || out_dtype == K3CUDA_BF16, "bad out_dtype");
    K3_ARG_CHECK(H >= 1 && H <= MLA_HP && B >= 0 && cap >= 1, "bad H=%d B=%d cap=%d", H, B, cap);
    if (B == 0) return K3CUDA_OK;
    K3_ARG_CHECK(ctx_lens, "null ctx_lens");
    for (int b = 0; b < B; b++)
        K3_ARG_CHECK(ctx_lens[b] >= 1 && ctx_lens[b] <= cap, "ctx_lens[%d]=%d outside [1, %d]", b,
                     ctx_lens[b], cap);
    K3_ARG_CHECK(out && q_nope && q_rope && latent && rope && w_uk && w_uv, "null pointer");
    K3_ARG_CHECK(aligned(latent, 16) && aligned(rope, 16), "caches must be 16-byte aligned");
    K3_ARG_CHECK((long long)B * cap < (1ll << 31) && (long long)B * MLA_HP < (1ll << 31),
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
    __nv_bfloat16 *qlat = (__nv_bfloat16 *)w;
    w += align256((size_t)B * MLA_HP * MLA_QW * 2);
    float *part = (float *)w;
    K3_CUDA_TRY(cudaMemcpyAsync(d_segs, p.segs.data(), (size_t)nseg * sizeof(MlaSeg),
                                cudaMemcpyHostToDevice, ctx->stream));
    K3_CUDA_TRY(cudaMemcpyAsync(d_cl, p.cl_begin.data(), p.cl_begin.size() * sizeof(int),
                                cudaMemcpyHostToDevice, ctx->stream));
    K3_CUDA_TRY(cudaMemcpyAsync(d_slot0, p.slot0.data(), ((size_t)B + 1) * sizeof(int),
                                cudaMemcpyHostToDevice, ctx->stream));
    K3_CUDA_TRY(cudaMemcpyAsync(d_lens, ctx_lens, (size_t)B * sizeof(int), cudaMemcpyHostToDevice,
                                ctx->stream));

    MlaMaps maps;
    rc = make_tmap_2d(&maps.q, qlat, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, MLA_QW,
                      (uint64_t)B * MLA_HP, MLA_QW * 2, 64, MLA_HP);
    if (!rc)
        rc = make_tmap_2d(&maps.lat, latent, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, MLA_DL,
                          (uint64_t)B * cap, MLA_DL * 2, 64, MLA_TILE);
    if (!rc)
        rc = make_tmap_2d(&maps.rope, rope, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, MLA_DR,
                          (uint64_t)B * cap, MLA_DR * 2, 64, MLA_TILE);
    if (rc) return rc;

    mla_q_absorb<<<dim3(MLA_HP, (B + 15) / 16), 256, 0, ctx->stream>>>(
        (const __nv_bfloat16 *)q_nope, (const __nv_bfloat16 *)q_rope,
        (const __nv_bfloat16 *)w_uk, qlat, B, H);
    rc = after_launch(ctx, "mla_q_absorb");
    if (rc) return rc;

    K3_CUDA_TRY(cudaFuncSetAttribute(mla_attend_tc, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     MLA_SMEM));
    const float scale_log2e = scale * 1.4426950408889634f;
    mla_attend_tc<<<2 * p.ncl, 192, MLA_SMEM, ctx->stream>>>(maps, d_segs, d_cl, d_lens, part, H,
                                                           cap, scale_log2e, ctx->err_word);
    rc = after_launch(ctx, "mla_attend_tc");
    if (rc) return rc;

    const size_t msmem = ((size_t)nseg + 64 * 65 + 128 * 65) * sizeof(float);
    if (out_dtype == K3CUDA_BF16) {
        K3_CUDA_TRY(cudaFuncSetAttribute(mla_merge_project<__nv_bfloat16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem));
        mla_merge_project<__nv_bfloat16><<<H, 256, msmem, ctx->stream>>>(
            part, d_slot0, (const __nv_bfloat16 *)w_uv, (__nv_bfloat16 *)out, B, H, nseg);
    } else {
        K3_CUDA_TRY(cudaFuncSetAttribute(mla_merge_project<float>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)msmem));
        mla_merge_project<float><<<H, 256, msmem, ctx->stream>>>(
            part, d_slot0, (const __nv_bfloat16 *)w_uv, (float *)out, B, H, nseg);
    }
    return after_launch(ctx, "mla_merge_project");
}
