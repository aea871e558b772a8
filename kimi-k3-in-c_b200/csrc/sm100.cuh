// sm100.cuh -- thin inline-PTX layer over the Blackwell (sm_100a) asynchronous units used by
// the tensor-core kernels: mbarriers, TMA tensor loads, Tensor Memory (TMEM) allocation and
// access, tcgen05.mma with shared-memory descriptors, and cluster shared memory.
//
// Conventions
//   * Shared-memory operands use the 128-byte swizzle (SW128): a tile row is 64 bf16 (or
//     32 fp32) = 128 B, eight rows form a 1024-byte swizzle atom, and every tile starts on a
//     1024-byte boundary so the descriptor's base offset is 0.
//   * K-major operand (K contiguous, the TMA box inner dimension): atoms are stacked along
//     M/N every 1024 B (SBO); a K step of 32 bytes inside the atom advances the start
//     address by 32 B; the next 64-element K block is a separate [rows x 128 B] region.
//   * MN-major operand (M/N contiguous): an atom covers 64 M/N values x 8 K rows; atoms are
//     stacked along K every 1024 B (SBO) and along M/N by LBO bytes.
//   * Every wait is bounded: a wait that does not complete within the context's bound
//     (k3cuda_set_wait_limit; 2^31 SM cycles, about a second, by default) records `code` in
//     the kernel's error word and returns false, and the kernel
//     then skips the rest of its work, waits (bounded) for its own copies, frees TMEM and
//     exits. No wait can hang the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace k3 {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// 2^x on the special-function unit (ex2.approx, flushes subnormal results to zero).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ------------------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Arrive on the mbarrier at the same shared offset in cluster CTA `cta` (release at
// cluster scope, so the arriving thread's earlier shared::cluster stores are visible to a
// waiter that acquires at cluster scope).
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t *bar, uint32_t cta) {
    asm volatile(
        "{\n\t.reg .b32 ra;\n\t"
        "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
        "mbarrier.arrive.release.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
        "r"(cta)
        : "memory");
}

// Relaxed remote arrive: for signals that order no data of this thread's (e.g. "I have
// finished reading your buffer": the reads are complete once their values are consumed).
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint64_t *bar, uint32_t cta) {
    asm volatile(
        "{\n\t.reg .b32 ra;\n\t"
        "mapa.shared::cluster.u32 ra, %0, %1;\n\t"
        "mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [ra];\n\t}" ::"r"(smem_u32(bar)),
        "r"(cta)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

constexpr long long kWaitCycles = 1ll << 31;

// The error block of a context (256 bytes of device memory): word 0 holds the code of the
// first wait that gave up, the 64-bit value at byte 8 the bound of every wait in SM clock
// cycles (k3cuda_set_wait_limit; kWaitCycles, about a second, when it is not positive).
__device__ __forceinline__ long long wait_limit(const unsigned *err) {
    const long long lim = *(const volatile long long *)(err + 2);
    return lim > 0 ? lim : kWaitCycles;
}

// Bounded wait; on timeout records `code` in *err (first error wins) and returns false.
// try_wait blocks in hardware for a while before returning false, so the loop spins slowly;
// the error word (another role's timeout) and the clock are only checked every 64 tries,
// which keeps a global load off the fast path.
template <bool kCluster>
__device__ __forceinline__ bool mbar_wait_impl(uint64_t *bar, uint32_t parity, unsigned *err,
                                               unsigned code) {
    if (kCluster ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    const long long lim = wait_limit(err);
    for (uint32_t i = 1;; i++) {
        if (kCluster ? mbar_try_wait_cluster(bar, parity) : mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*(volatile unsigned *)err) return false;
            if (clock64() - t0 > lim) {
                atomicCAS(err, 0u, code);
                return false;
            }
        }
    }
}

__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned *err,
                                          unsigned code) {
    return mbar_wait_impl<false>(bar, parity, err, code);
}

__device__ __forceinline__ bool mbar_wait_cluster(uint64_t *bar, uint32_t parity, unsigned *err,
                                                  unsigned code) {
    return mbar_wait_impl<true>(bar, parity, err, code);
}

// Bounded wait by a whole warp; true only if every lane's wait completed.
__device__ __forceinline__ bool warp_wait_all(uint64_t *bar, uint32_t parity, unsigned *err,
                                              unsigned code) {
    const bool ok = mbar_wait(bar, parity, err, code);
    return __all_sync(0xffffffffu, ok);
}

// Bounded wait that reports nothing (used only to drain a CTA's own loads on exit).
__device__ __forceinline__ bool mbar_wait_quiet(uint64_t *bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitCycles) return false;
    return true;
}

// ------------------------------------------------------------------ SW128 tiles, bf16
// byte offset of the 16-byte chunk `c` (0..7) of row `r` in a 128-byte-swizzled tile whose
// base is 1024-byte aligned
__device__ __forceinline__ uint32_t swz(int r, int c) {
    return (uint32_t)(r * 128 + (((c ^ r) & 7) << 4));
}
// byte offset of bf16 element (r, c), c < 64, of such a tile
__device__ __forceinline__ uint32_t swz_elem(int r, int c) {
    return swz(r, c >> 3) + (uint32_t)(c & 7) * 2;
}

__device__ __forceinline__ uint32_t pack_bf2(float a, float b) {
    const __nv_bfloat162 p = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&p);
}
__device__ __forceinline__ uint4 pack_bf8(const float *v) {
    return make_uint4(pack_bf2(v[0], v[1]), pack_bf2(v[2], v[3]), pack_bf2(v[4], v[5]),
                      pack_bf2(v[6], v[7]));
}
__device__ __forceinline__ void unpack_bf8(uint4 u, float *v) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; i++) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
__device__ __forceinline__ void st16s(uint8_t *p, uint4 v) { *reinterpret_cast<uint4 *>(p) = v; }

// ------------------------------------------------------------------------------ TMA
// Untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global
// memory into this CTA's shared memory, completing on `bar` (transaction bytes).
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled load of box (c0 = inner, c1 = outer) into shared memory, completing on `bar`
// (transaction bytes). The destination is this CTA's own shared memory.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int c0, int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// 3-D tiled store of a shared-memory box (same layout as the load) to global memory, as part
// of this thread's current bulk group. Coordinates must be non-negative.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int c0,
                                             int c1, int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
            (uint64_t)map),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's committed bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Bring a box into L2 ahead of its load (no shared memory, no completion to wait for).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap *map, int c0, int c1) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                     (uint64_t)map),
                 "r"(c0), "r"(c1)
                 : "memory");
}
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap *map, int c0, int c1, int c2) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     (uint64_t)map),
                 "r"(c0), "r"(c1), "r"(c2)
                 : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy (tcgen05.mma, TMA).
__device__ __forceinline__ void fence_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------------------- TMEM
// Allocate `ncols` (power of two >= 32) columns; the base address is written to *dst
// (shared memory). Must be executed by one full warp.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns: thread t of the warp receives lane
// (warp%4)*32 + t of the address's lane quarter.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// As tmem_ld16, 32 consecutive columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float *v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// ----------------------------------------------------------------------- descriptors
constexpr uint32_t kSw128 = 2;  // layout type: 128-byte swizzle

// Shared-memory matrix descriptor (start, leading and stride byte offsets, SW128).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | ((uint64_t)kSw128 << 61);
}

// K-major SW128 operand at `saddr` (1024-aligned region of rows x 128 B): the K step of
// 16 bf16 (or 8 tf32) is +32 B on the start address.
__device__ __forceinline__ uint64_t sdesc_kmajor(uint32_t saddr) { return sdesc(saddr, 16, 1024); }

// MN-major SW128 operand: `mn_stride` bytes between consecutive 64-wide M/N blocks.
__device__ __forceinline__ uint64_t sdesc_mnmajor(uint32_t saddr, uint32_t mn_stride) {
    return sdesc(saddr, mn_stride, 1024);
}

// Instruction descriptor, kind::f16 with bf16 A/B and fp32 D (or kind::tf32 with tf32
// A/B when tf32 is true).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool a_mn, bool b_mn,
                                                 bool tf32 = false) {
    return (1u << 4) | ((tf32 ? 2u : 1u) << 7) | ((tf32 ? 2u : 1u) << 10) |
           ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] . B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] . B[smem]^T (A K-major in TMEM: row m in lane m, two bf16 per
// 32-bit column, K ascending), issued by one thread.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// ---------------------------------------------------------------------------- cluster
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}

// Address of the same shared location in cluster CTA `cta`.
__device__ __forceinline__ uint32_t map_peer(uint32_t saddr, uint32_t cta) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(cta));
    return r;
}

__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b),
                 "f"(c), "f"(d)
                 : "memory");
}

// Asynchronous 16-byte store into cluster CTA shared memory that completes `bytes`
// transactions on the mbarrier `rbar` of the destination CTA (both addresses from map_peer).
__device__ __forceinline__ void st_async_v4(uint32_t raddr, float a, float b, float c, float d,
                                            uint32_t rbar) {
    asm volatile(
        "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::
            "r"(raddr), "f"(a), "f"(b), "f"(c), "f"(d), "r"(rbar)
        : "memory");
}

// Barrier among `nthreads` threads (a multiple of 32) on hardware barrier `id` (1..15).
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace sm100
}  // namespace k3
