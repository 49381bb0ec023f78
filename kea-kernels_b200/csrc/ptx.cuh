// ptx.cuh - inline-PTX helpers for sm_100a: mbarriers, TMA / bulk copies, tcgen05 (TMEM, MMA), clusters.
// Written against the public PTX ISA (sm_100a). Every wait on an mbarrier is bounded by a clock budget so a
// kernel can report a timeout instead of hanging the GPU.
#pragma once

#include <cstdint>
#include <cuda.h>

namespace kea {

#define KEA_DEVI __device__ __forceinline__

KEA_DEVI uint32_t smem_u32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// ---- mbarrier ------------------------------------------------------------------------------------------
KEA_DEVI void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
KEA_DEVI void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
KEA_DEVI void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Tests phase `parity`; when it is not complete the thread is suspended in hardware (up to ~1 ms) until it
// completes, instead of spinning and taking issue slots from the warps that do the work.
KEA_DEVI bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(1000000u)
        : "memory");
    return done != 0;
}
// Non-blocking test of phase `parity` (no suspension): the cheap first look of every wait.
KEA_DEVI bool mbar_peek(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}
// Waits for phase `parity` of the barrier; false when `budget` SM clocks pass first.
KEA_DEVI bool mbar_wait(uint32_t bar, uint32_t parity, long long budget) {
    if (mbar_peek(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_test(bar, parity)) {
        if (clock64() - start > budget) return false;
    }
    return true;
}
// For long waits of warps that have nothing else to do (an epilogue waiting for a whole main loop): between tests the
// warp sleeps `ns` nanoseconds, so its polling takes no issue slots or shared-memory cycles from the working warps.
KEA_DEVI bool mbar_wait_sleep(uint32_t bar, uint32_t parity, long long budget, uint32_t ns) {
    if (mbar_test(bar, parity)) return true;
    const long long start = clock64();
    while (true) {
        __nanosleep(ns);
        if (mbar_test(bar, parity)) return true;
        if (clock64() - start > budget) return false;
    }
}
KEA_DEVI void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory writes before later async-proxy (TMA / tcgen05) accesses.
KEA_DEVI void fence_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// orders this thread's generic-proxy global accesses with later async-proxy (TMA) accesses
KEA_DEVI void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// One lane of the (converged) warp gets true: elect.sync, which lets the compiler keep warp-uniform operands of the
// elected lane's instructions in uniform registers.
KEA_DEVI bool elect_one() {
    uint32_t pred;
    asm volatile("{\n\t.reg .pred P1;\n\telect.sync _|P1, 0xffffffff;\n\tselp.b32 %0, 1, 0, P1;\n\t}\n" : "=r"(pred));
    return pred != 0;
}

// ---- copies into shared memory ----------------------------------------------------------------------------
// 3-D tiled TMA load (no multicast) completing on an mbarrier of this CTA.
KEA_DEVI void tma_load_3d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];"
        ::"r"(dst), "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}
// 2-D and 4-D tiled TMA loads (no multicast).
KEA_DEVI void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];"
        ::"r"(dst), "l"(map), "r"(bar), "r"(x), "r"(y)
        : "memory");
}
KEA_DEVI void tma_load_4d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y, int z, int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], [%2];"
        ::"r"(dst), "l"(map), "r"(bar), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}
// Untiled bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
KEA_DEVI void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}
// 2-D tiled TMA store shared -> global (bulk-group completion; out-of-range rows / columns are not written).
KEA_DEVI void tma_store_2d(const CUtensorMap *map, uint32_t src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
                 ::"l"(map), "r"(src), "r"(x), "r"(y)
                 : "memory");
}
KEA_DEVI void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
KEA_DEVI void bulk_wait_group_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// At most one committed bulk group may still be reading its shared-memory source.
KEA_DEVI void bulk_wait_group_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
KEA_DEVI void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
KEA_DEVI void prefetch_tensormap(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ---- tcgen05: tensor memory and the 5th-generation MMA -------------------------------------------------------
KEA_DEVI void tmem_alloc(uint32_t slot, uint32_t cols) {  // whole warp
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(cols) : "memory");
}
KEA_DEVI void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
KEA_DEVI void tmem_dealloc(uint32_t taddr, uint32_t cols) {  // whole warp
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
KEA_DEVI void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
KEA_DEVI void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, signed INT8 inputs, INT32 accumulators.
KEA_DEVI void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives once on `bar` when every tcgen05.mma this thread issued before it has completed.
KEA_DEVI void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i).
KEA_DEVI void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
KEA_DEVI void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// tcgen05.ld fills its destination registers asynchronously, but to the compiler they are written when the load
// statement executes: arithmetic on them could be scheduled above tcgen05.wait::ld and read registers that have not
// landed. After the wait, this empty volatile statement (ordered after it, as every volatile asm) rewrites the
// registers, so each later use depends on a statement that follows the wait.
KEA_DEVI void tmem_regs_ready(uint32_t (&r)[16]) {
    asm volatile(""
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
                 :
                 : "memory");
}
KEA_DEVI void tmem_regs_ready(uint32_t (&r)[32]) {
    tmem_regs_ready(*reinterpret_cast<uint32_t(*)[16]>(&r[0]));
    tmem_regs_ready(*reinterpret_cast<uint32_t(*)[16]>(&r[16]));
}

// Shared-memory matrix descriptor of a K-major operand stored in the 128-byte swizzle layout:
// rows of 128 bytes, 8-row (1024 B) swizzle atoms stacked along M/N (stride 1024 B), atom base 1024-aligned.
// Fields: start address >> 4 [0,14), leading byte offset >> 4 [16,30) (unused for this layout: 1),
// stride byte offset >> 4 [32,46), version 1 [46,48), layout type 2 = 128-byte swizzle [61,64).
KEA_DEVI uint64_t sw128_kmajor_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::i8: D = S32 [4,6), A = B = signed 8-bit [7,10) / [10,13), both K-major,
// N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_i8(uint32_t m, uint32_t n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// ---- clusters ----------------------------------------------------------------------------------------------
KEA_DEVI uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
KEA_DEVI void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
KEA_DEVI void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
KEA_DEVI void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
KEA_DEVI uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
KEA_DEVI int ld_cluster_s32(uint32_t addr) {
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}

// Cluster barrier without .aligned: legal when the warps of a CTA reach it from different code paths.
KEA_DEVI void cluster_sync_relaxed_paths() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

// ---- CTA pairs (tcgen05 cta_group::2) -------------------------------------------------------------------------
// Every tcgen05 instruction of a pair kernel uses cta_group::2. One warp of EACH CTA of the pair (the same warp
// index in both) allocates and frees; the allocation covers the same columns in both CTAs' tensor memory.
KEA_DEVI void tmem_alloc_pair(uint32_t slot, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot), "r"(cols) : "memory");
}
KEA_DEVI void tmem_relinquish_pair() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
KEA_DEVI void tmem_dealloc_pair(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
// Issued by the even CTA of the pair: D (M = 256 rows: rows 0-127 in the even CTA's tensor memory, 128-255 in the
// odd CTA's) (+)= A (rows 0-127 from the even CTA's shared memory, 128-255 from the odd CTA's, at the same offset)
// x B^T (N / 2 rows from each CTA's shared memory, at the same offset). Signed INT8, INT32 accumulators.
KEA_DEVI void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrives once on the mbarrier at shared-memory offset `bar` in every CTA of `cta_mask` when the pair MMAs this
// thread issued before it have completed (a tcgen05 completion signal; it moves no data).
KEA_DEVI void mma_commit_pair(uint32_t bar, uint16_t cta_mask) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(bar), "h"(cta_mask)
                 : "memory");
}
// Arrive on an mbarrier given by its shared::cluster address (own CTA or a peer), with the instruction's default
// semantics (release at CTA scope). A cluster-scope release here waits for every outstanding memory operation of the
// thread and cost about 1 us per arrival in the pair kernel's pipeline; the data this arrival publishes is in the
// arriving CTA's own shared memory, made visible to the tensor cores by fence.proxy.async before the arrival.
KEA_DEVI void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// Like mbar_test / mbar_wait, with acquire at cluster scope (the phase was completed by arrivals from a peer CTA).
KEA_DEVI bool mbar_test_cluster(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(done)
        : "r"(bar), "r"(parity), "r"(1000000u)
        : "memory");
    return done != 0;
}
KEA_DEVI bool mbar_wait_cluster(uint32_t bar, uint32_t parity, long long budget) {
    if (mbar_test_cluster(bar, parity)) return true;
    const long long start = clock64();
    while (!mbar_test_cluster(bar, parity)) {
        if (clock64() - start > budget) return false;
    }
    return true;
}

// ---- programmatic dependent launch --------------------------------------------------------------------------
KEA_DEVI void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
KEA_DEVI void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- exact FP32 epilogue pieces ------------------------------------------------------------------------------
// SiLU as y / (2^(-y * log2(e)) + 1) with the hardware ex2.approx and div.full instructions, the instruction
// sequence the kea-kernels epilogue uses for its activation.
KEA_DEVI float silu_approx(float y) {
    float e, r;
    const float t = __fmul_rn(-y, 1.4426950408889634f);
    asm("ex2.approx.f32 %0, %1;" : "=f"(e) : "f"(t));
    const float d = __fadd_rn(e, 1.0f);
    asm("div.full.f32 %0, %1, %2;" : "=f"(r) : "f"(y), "f"(d));
    return r;
}

}  // namespace kea
