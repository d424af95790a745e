// Minimal sm_100a tensor-core toolkit: tcgen05.mma (kind::f16, bf16 inputs,
// fp32 accumulators in TMEM), shared-memory matrix descriptors for the
// K-major no-swizzle canonical layout, TMEM allocation and loads, mbarriers.
//
// Canonical K-major SWIZZLE_NONE operand layout used by every kernel here:
// the tile is cut into 8-row x 16-byte "core matrices" (8 bf16 along K);
// element (r, k) of a tile with K columns sits at byte
//     (r / 8) * SBO + (k / 8) * 128 + (r % 8) * 16 + (k % 8) * 2,
// with LBO = 128 B (next core matrix along K) and SBO = 16 * K bytes (next
// 8-row group).  One MMA consumes K = 16 (two core matrices along K); the
// descriptor for k-step s starts at byte offset s * 256.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define TC_DEV __device__ __forceinline__

TC_DEV uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// byte offset of element (r, k) in a canonical K-major tile with K columns
TC_DEV uint32_t canon_off(int r, int k, int K) {
    return (uint32_t)((r >> 3) * (16 * K) + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2);
}

// byte offset of element (mn, k) in a canonical MN-major no-swizzle tile with
// MN extent M: 8 consecutive MN elements form a 16-byte core-matrix row, 8 K
// rows make a 128-byte core matrix; MN groups are adjacent (SBO = 128 B) and
// K groups of 8 are LBO = 16 * M bytes apart.
TC_DEV uint32_t canon_off_mn(int mn, int k, int M) {
    return (uint32_t)((mn >> 3) * 128 + (k >> 3) * (16 * M) + (k & 7) * 16 + (mn & 7) * 2);
}

// Shared-memory matrix descriptor (sm_100 format, version 1, no swizzle).
TC_DEV uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;            // version
    return d;                          // base offset 0, lbo mode 0, layout 0 (no swizzle)
}

// Instruction descriptor: D fp32, A/B bf16, M x N; a_mn / b_mn select the
// MN-major layout for that operand (default K-major).
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, int a_mn = 0, int b_mn = 0) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
           ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

TC_DEV void tc_mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        :
        : "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}

TC_DEV void tc_commit(uint64_t* mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(mbar)) : "memory");
}

// whole warp: allocate ncols TMEM columns, address written to *slot (smem)
TC_DEV void tc_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

TC_DEV void tc_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 :: "r"(taddr), "r"(ncols) : "memory");
}

TC_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
TC_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// make generic-proxy shared-memory writes visible to the tensor core
TC_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 lanes x 32 bits, 16 consecutive columns per thread
TC_DEV void tc_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

TC_DEV void mbar_init(uint64_t* mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(mbar)), "r"(count)
                 : "memory");
}

// Bounded wait for phase `parity` of an mbarrier.  Returns false when the
// iteration limit ran out (the caller records an error and exits cleanly).
TC_DEV bool mbar_wait(uint64_t* mbar, uint32_t parity, uint32_t limit = (1u << 26)) {
    const uint32_t a = smem_u32(mbar);
    for (uint32_t it = 0; it < limit; ++it) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(ok) : "r"(a), "r"(parity) : "memory");
        if (ok) return true;
    }
    return false;
}

// split an fp32 value into bf16 hi + bf16 lo (x ~= hi + lo to ~2^-17 relative)
TC_DEV void split_bf16(float x, uint16_t& hi, uint16_t& lo) {
    const __nv_bfloat16 h = __float2bfloat16_rn(x);
    const float r = x - __bfloat162float(h);
    hi = __bfloat16_as_ushort(h);
    lo = __bfloat16_as_ushort(__float2bfloat16_rn(r));
}

// TMA bulk copy (non-tensor) global -> shared, completion counted in bytes
// on an mbarrier.  Both addresses 16-byte aligned, size a multiple of 16.
TC_DEV void mbar_expect_tx(uint64_t* mbar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_u32(mbar)), "r"(bytes) : "memory");
}
TC_DEV void bulk_g2s(void* dst_smem, const void* src_gmem, uint32_t bytes, uint64_t* mbar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        :: "r"(smem_u32(dst_smem)), "l"(src_gmem), "r"(bytes), "r"(smem_u32(mbar)) : "memory");
}

// 16-byte asynchronous global -> shared copy (L2 only), and an arrival on an
// mbarrier once all of this thread's earlier asynchronous copies completed
// (noinc: the arrival counts toward the barrier's initial count)
TC_DEV void cp_async16(void* dst_smem, const void* src_gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
                 :: "r"(smem_u32(dst_smem)), "l"(src_gmem) : "memory");
}
TC_DEV void cp_async_arrive_noinc(uint64_t* mbar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];"
                 :: "r"(smem_u32(mbar)) : "memory");
}

// TMA tensor copy of one 2-D box (coordinates x = innermost) into shared
// memory, completion counted on an mbarrier.  No multicast.
TC_DEV void tma_load_2d(uint32_t dst, const void* map, int x, int y, uint64_t* mbar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];"
        :: "r"(dst), "l"(map), "r"(x), "r"(y), "r"(smem_u32(mbar)) : "memory");
}

TC_DEV void mbar_arrive(uint64_t* mbar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(mbar)) : "memory");
}

// 128-byte-swizzle shared-memory descriptor (layout type 2 in bits 61-63):
// K-major tiles of 128-byte rows in 8-row / 1024-byte atoms as written by a
// TMA copy with CU_TENSOR_MAP_SWIZZLE_128B into a 1024-byte aligned buffer.
TC_DEV uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return smem_desc(saddr, lbo, sbo) | ((uint64_t)2 << 61);
}

// named barrier over a subset of the CTA's warps
TC_DEV void named_bar(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

// 32 lanes x 32 bits, 8 consecutive columns per thread
TC_DEV void tc_ld8(uint32_t taddr, float* v) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// TMA tensor store of one 2-D box from shared memory (bulk-group completion)
TC_DEV void tma_store_2d(const void* map, int x, int y, uint32_t src) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
        :: "l"(map), "r"(x), "r"(y), "r"(src) : "memory");
}
TC_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until the committed bulk stores have finished reading shared memory
TC_DEV void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// wait until the committed bulk stores are complete (globally visible)
TC_DEV void bulk_wait0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }


// 32 lanes x 32 bits, 4 consecutive columns per thread
TC_DEV void tc_ld4(uint32_t taddr, float* v) {
    uint32_t r[4];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

// L2 eviction-priority policies for TMA copies of streamed data
TC_DEV uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
TC_DEV void tma_load_2d_hint(uint32_t dst, const void* map, int x, int y, uint64_t* mbar,
                             uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3}], [%4], %5;"
        :: "r"(dst), "l"(map), "r"(x), "r"(y), "r"(smem_u32(mbar)), "l"(policy) : "memory");
}
TC_DEV void tma_store_2d_hint(const void* map, int x, int y, uint32_t src, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2}], [%3], %4;"
        :: "l"(map), "r"(x), "r"(y), "r"(src), "l"(policy) : "memory");
}

// ---------------------------------------------------------------------------
// CTA-pair (cta_group::2) helpers: one tcgen05.mma spans the tensor cores of
// two SMs of a cluster of 2; each CTA holds half of A (its 128 rows) and half
// of B in its own shared memory, and its 128 accumulator rows in its own TMEM.
// ---------------------------------------------------------------------------
TC_DEV uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of a shared::cta location in CTA `rank` of the cluster
TC_DEV uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
TC_DEV void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
                 ::: "memory");
}
// arrive (with transaction bytes expected) on an mbarrier given by its cluster address
TC_DEV void mbar_arrive_expect_tx_cl(uint32_t cl_addr, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;"
                 :: "r"(cl_addr), "r"(bytes) : "memory");
}
TC_DEV void mbar_arrive_cl(uint32_t cl_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" :: "r"(cl_addr) : "memory");
}
// TMA tensor load into this CTA's shared memory whose completion is counted
// on the pair leader's mbarrier (cluster address).  No multicast.
TC_DEV void tma_load_2d_pair(uint32_t dst, const void* map, int x, int y, uint32_t mbar_cl) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];"
        :: "r"(dst), "l"(map), "r"(x), "r"(y), "r"(mbar_cl) : "memory");
}
TC_DEV void tc_mma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n"
        :
        : "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
// arrive on the mbarrier at this shared offset in every CTA of cta_mask when
// the pair's issued MMAs have completed
TC_DEV void tc_commit_pair(uint64_t* mbar, uint16_t cta_mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
        :: "r"(smem_u32(mbar)), "h"(cta_mask) : "memory");
}
// one warp in each CTA of the pair (same warp index): TMEM for both
TC_DEV void tc_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
TC_DEV void tc_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;"
                 :: "r"(taddr), "r"(ncols) : "memory");
}
