// gemm_pair_kernel.cuh - the large-M low-bit GEMM for sm_100a: a persistent kernel on CTA pairs (tcgen05
// cta_group::2), one INT8 activation part.
//
// A pair tile is 256 tokens x 256 channels. The even CTA of a thread-block cluster of two holds tokens 0-127 of the
// tile and channel rows 0-127 (one panel tile); the odd CTA holds tokens 128-255 and channel rows 128-255. Each CTA
// loads its own activation box and packed codes and expands its own half of the weights, so the tensor cores of
// both SMs read only their own shared memory, and every expanded weight serves 256 tokens while each SM stores only
// half of the B operand: per K = 32 step an SM reads 4 KB of activations + 4 KB of weights for 128 x 256 x 32 MACs,
// which keeps shared memory under its bandwidth at the INT8 rate. The even CTA issues tcgen05.mma.cta_group::2
// (M = 256, N = 256) for both; each CTA's tensor memory receives its 128 token rows x 256 channels.
//
// The pairs walk the tile list persistently (pair p takes tiles p, p + pairs, ...). Tensor memory holds two
// 256-column accumulator buffers, so the epilogue of tile i (8 warps per CTA) runs while the MMAs of tile i + 1
// accumulate into the other buffer.
//
// Warps per CTA (576 threads):
//   warp 0       producer: per k-block one TMA box of activations (128 tokens x 128 k, 128-byte swizzle) and one bulk
//                copy of the packed codes (128 channel rows x 128 k), on this CTA's `full` barrier;
//   warp 1       allocates tensor memory for the pair; in the even CTA one elected lane issues the MMAs, frees each
//                stage in both CTAs (tcgen05.commit to both CTAs' `empty`) and hands finished accumulators to both
//                CTAs' epilogues (`acc_full`);
//   warps 2-9    epilogue: TMEM -> comb_1 * alpha (+ bias) (SiLU) -> FP32 / FP16, staged in shared memory and written
//                with TMA stores; then release the buffer (`acc_empty` of the even CTA, 16 warp arrivals);
//   warps 10-17  expanders, two groups of four warps taking alternate k-blocks: packed codes -> INT8 +-1 / -1 0 +1 in
//                the 128-byte-swizzled K-major B tile, then arrive on the even CTA's `ready` barrier (8 warp arrivals:
//                the stage is complete in both CTAs).
// Every wait is bounded (kWaitBudget); on expiry the kernel reports KEA_DEVERR_TIMEOUT, lets its copies and MMAs
// drain, and returns.
#pragma once

#include "gemm_kernel.cuh"

namespace kea {

constexpr int kPairWarps = 18;
constexpr int kPairThreads = kPairWarps * 32;     // 576
constexpr int kPairTileM = 256;                   // tokens per pair tile (128 per CTA)
constexpr int kPairTileN = 256;                   // channels per pair tile (one 128-row panel tile per CTA)
constexpr int kPairEpiWarp0 = 2, kPairEpiWarps = 8;
constexpr int kPairExpWarp0 = 10, kPairExpWarps = 8;
constexpr int kPairExpGroups = 2, kPairExpGroupWarps = kPairExpWarps / kPairExpGroups;
constexpr int kPairMaxStages = 8;
constexpr uint32_t kPairAccCols = 256;            // one accumulator buffer: 128 lanes x 256 INT32 columns
constexpr uint32_t kPairTmemCols = 512;           // two buffers
constexpr uint32_t kPairHalfTile = 16384;         // 128 rows x 128 bytes: one CTA's activation or B tile per stage
constexpr uint32_t kPairStageOut = 2048;          // epilogue staging: one TMA box of 32 rows x 64 bytes, two per warp
constexpr uint32_t kPairStagingBytes = kPairEpiWarps * 2 * kPairStageOut;   // 32 KB
constexpr uint32_t kPairChannelBytes = kPairEpiWarps * 1024;                // alpha + bias of each warp's 128 channels

struct PairArgs {
    const uint8_t *panels;
    const float *qs;             // FP32 [m] token scales
    const float *alpha;          // FP32 [n]
    const float *bias;           // FP32 [n] or null
    int *acc;                    // optional INT32 [m][ld_acc]
    long long ld_acc;
    int M, N, K, kb_total;
    int n_tiles, tiles;          // 256-channel tiles, pair tiles in all
    int flags;                   // KEA_FLAG_SILU
    int pdl;
    int y_f16;
    int stages;
    uint32_t *err;
};

// Per-step timestamps of the first pair (SM clocks since each CTA's start) for latency studies: compiled in only
// with -DKEA_TRACE and read back by kea_pair_trace_read. The default build has no trace code.
#ifdef KEA_TRACE
constexpr int kPairTraceEvents = 16, kPairTraceSteps = 64;
__device__ long long g_pair_trace[2][kPairTraceEvents][kPairTraceSteps];
__shared__ long long s_ptrace_clock0;
#define KEA_PTRACE(cond, ev, i)                                                                                   \
    do {                                                                                                          \
        if ((cond) && blockIdx.x < 2 && (i) < kPairTraceSteps)                                                    \
            g_pair_trace[blockIdx.x][ev][i] = clock64() - s_ptrace_clock0;                                        \
    } while (0)
#else
#define KEA_PTRACE(cond, ev, i) do { } while (0)
#endif

// INT32 -> FP32 for |a| < 2^22 (|acc| <= 127 K with K <= 32768 here): exact, so equal to cvt.rn.f32.s32, in two
// full-rate operations. 0x4B400000 is the bit pattern of 1.5 * 2^23, whose mantissa holds a + 2^22 exactly.
KEA_DEVI float int_to_float_exact(int a) { return __fsub_rn(__int_as_float(a + 0x4B400000), 12582912.0f); }

// comb_1, alpha / bias, optional SiLU: one IEEE FP32 rounding per operation (the reference's epilogue order).
KEA_DEVI float finish1(int acc, float s, float alpha, bool has_bias, float bias, int flags) {
    const float r = __fmul_rn(int_to_float_exact(acc), s);
    float y = has_bias ? __fmaf_rn(r, alpha, bias) : __fmul_rn(r, alpha);
    if (flags & 1) y = silu_approx(y);
    return y;
}

// One epilogue warp's share of a finished tile: its 32 token rows x 128 channels of tensor memory, in groups of
// 4 KB of output (64 FP16 or 32 FP32 channels). For each 32 columns of a group the warp loads them from TMEM and
// finishes them in registers (alpha / bias from the warp's shared-memory copy); before the group's first staging store
// it waits until the previous group's TMA stores have read the warp's 4 KB staging buffer; then it stages the rows
// (32 x 64-byte boxes, 64-byte swizzle as the store's tensor map), fences once and issues two TMA stores. After its
// last TMEM read the warp releases the accumulator buffer (`acc_empty`, a shared::cluster address).
template <bool F16, bool BIAS>
KEA_DEVI void pair_epilogue_tile(const PairArgs &a, const CUtensorMap *ymap, uint32_t cbase, uint32_t stg,
                                 uint32_t s_al, uint32_t s_bi, uint32_t acc_empty, int nbase, int trow0, int t, float sq) {
    constexpr int GROUP = F16 ? 64 : 32;     // channels per 4 KB group
    constexpr int CW = F16 ? 32 : 16;        // channels per 64-byte box row
    const int lane = threadIdx.x & 31;
#pragma unroll 1
    for (int c0 = 0; c0 < 128; c0 += GROUP) {
        KEA_PTRACE(threadIdx.x == kPairEpiWarp0 * 32, 10, c0 / GROUP);
#pragma unroll
        for (int h = 0; h < GROUP / 32; ++h) {
            const int c = c0 + 32 * h;
            uint32_t v[32];
            tmem_ld16(cbase + (uint32_t)c, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
            tmem_ld16(cbase + (uint32_t)(c + 16), *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
            tmem_wait_ld();
            if (c + 32 >= 128) {   // this warp's last read of the buffer: hand it back to the MMA warp
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(acc_empty);
            }
            if (a.acc && t < a.M) {
                int4 *dst = reinterpret_cast<int4 *>(a.acc + (long long)t * a.ld_acc + nbase + c);
#pragma unroll
                for (int q = 0; q < 8; ++q) dst[q] = make_int4((int)v[4 * q], (int)v[4 * q + 1], (int)v[4 * q + 2], (int)v[4 * q + 3]);
            }
            // finish in place: FP16 pairs packed into v[0 .. 16), FP32 bit patterns in v[0 .. 32)
#pragma unroll
            for (int jj = 0; jj < 32; jj += 4) {
                const uint4 alu = ld_shared_v4(s_al + (uint32_t)(c + jj) * 4u);
                uint4 biu = make_uint4(0u, 0u, 0u, 0u);
                if constexpr (BIAS) biu = ld_shared_v4(s_bi + (uint32_t)(c + jj) * 4u);
                const float f0 = finish1((int)v[jj], sq, __uint_as_float(alu.x), BIAS, __uint_as_float(biu.x), a.flags);
                const float f1 = finish1((int)v[jj + 1], sq, __uint_as_float(alu.y), BIAS, __uint_as_float(biu.y), a.flags);
                const float f2 = finish1((int)v[jj + 2], sq, __uint_as_float(alu.z), BIAS, __uint_as_float(biu.z), a.flags);
                const float f3 = finish1((int)v[jj + 3], sq, __uint_as_float(alu.w), BIAS, __uint_as_float(biu.w), a.flags);
                if constexpr (F16) {
                    v[jj / 2] = pack_half2(f0, f1);
                    v[jj / 2 + 1] = pack_half2(f2, f3);
                } else {
                    v[jj] = __float_as_uint(f0);
                    v[jj + 1] = __float_as_uint(f1);
                    v[jj + 2] = __float_as_uint(f2);
                    v[jj + 3] = __float_as_uint(f3);
                }
            }
            if (h == 0) {   // the previous group's stores must have read the staging buffer
                if (lane == 0) bulk_wait_group_read0();
                __syncwarp();
            }
            // FP16: these 32 channels are box h; FP32: boxes 0 and 1 (16 channels each)
#pragma unroll
            for (int b = 0; b < (F16 ? 1 : 2); ++b) {
                const uint32_t box = stg + (uint32_t)(F16 ? h : b) * kPairStageOut;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t off = (uint32_t)lane * 64u + (uint32_t)q * 16u;
                    const int w0 = b * 16 + q * 4;
                    st_shared_v4(box + (off ^ (((off >> 7) & 3u) << 4)), v[w0], v[w0 + 1], v[w0 + 2], v[w0 + 3]);
                }
            }
        }
        fence_async_shared();
        __syncwarp();
        if (lane == 0) {
            tma_store_2d(ymap, stg, nbase + c0, trow0);
            tma_store_2d(ymap, stg + kPairStageOut, nbase + c0 + CW, trow0);
            bulk_commit_group();
        }
        KEA_PTRACE(threadIdx.x == kPairEpiWarp0 * 32, 14, c0 / GROUP);
    }
}

template <int WBITS>
__global__ void __launch_bounds__(kPairThreads, 1) lowbit_gemm_pair_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                          const __grid_constant__ CUtensorMap ymap,
                                                                          const PairArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t bar_full[kPairMaxStages];    // this CTA's stage landed (TMA box + codes)
    __shared__ __align__(8) uint64_t bar_ready[kPairMaxStages];   // even CTA: the stage is expanded in both CTAs
    __shared__ __align__(8) uint64_t bar_empty[kPairMaxStages];   // the pair's MMAs are done with the stage
    __shared__ __align__(8) uint64_t bar_acc_full[2];             // accumulator buffer complete
    __shared__ __align__(8) uint64_t bar_acc_empty[2];            // even CTA: buffer drained by both epilogues
    __shared__ __align__(8) uint64_t bar_drain;                   // even CTA: every issued MMA has completed
    __shared__ uint32_t tmem_slot;

    constexpr uint32_t PKB = (uint32_t)WBITS * kPanelSubBytes;   // packed codes of one CTA per stage
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
    const uint32_t base = (smem_u32(dyn_smem) + 1023u) & ~1023u;
    const int S = a.stages;
    const uint32_t A0 = base, B0 = base + (uint32_t)S * kPairHalfTile, PK0 = base + 2u * (uint32_t)S * kPairHalfTile;
    const uint32_t STG0 = (PK0 + (uint32_t)S * PKB + 1023u) & ~1023u;
    const int kbt = a.kb_total;

#ifdef KEA_TRACE
    if (threadIdx.x == 0) {
        s_ptrace_clock0 = clock64();
        long long gt;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(gt));
        if (blockIdx.x < 2) g_pair_trace[blockIdx.x][7][0] = gt;
    }
#endif
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bar_full[s]), 1);
            mbar_init(smem_u32(&bar_ready[s]), 2 * kPairExpGroupWarps);
            mbar_init(smem_u32(&bar_empty[s]), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(smem_u32(&bar_acc_full[b]), 1);
            mbar_init(smem_u32(&bar_acc_empty[b]), 2 * kPairEpiWarps);
        }
        mbar_init(smem_u32(&bar_drain), 1);
        fence_barrier_init();
        prefetch_tensormap(&qmap);
        prefetch_tensormap(&ymap);
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(&tmem_slot), kPairTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();      // barrier initialisation and both CTAs' allocations are visible to the pair
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    KEA_PTRACE(threadIdx.x == 0, 7, 1);

    // With programmatic dependent launch, everything below may read what the previous kernel wrote.
    if (a.pdl) grid_dependency_wait();

    bool ok = true;
    if (warp == 0) {
        // ---------------- producer (one lane) ----------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            long long issued = 0;
            const uint32_t tx = kPairHalfTile + PKB;
            for (int tile = pair; tile < a.tiles && ok; tile += npairs) {
                const int mt = tile / a.n_tiles, nt = tile - mt * a.n_tiles;
                const int t0 = mt * kPairTileM + (int)rank * kBM;
                const uint8_t *wsrc = a.panels + (size_t)(nt * 2 + (int)rank) * (size_t)kbt * PKB;
                for (int kb = 0; kb < kbt; ++kb) {
                    if (issued >= S && !mbar_wait(smem_u32(&bar_empty[s]), ph ^ 1u, kWaitBudget)) {
                        ok = false;
                        break;
                    }
                    KEA_PTRACE(true, 0, issued);
                    const uint32_t full = smem_u32(&bar_full[s]);
                    mbar_arrive_expect_tx(full, tx);
                    tma_load_2d(A0 + (uint32_t)s * kPairHalfTile, &qmap, full, kb * kBK, t0);
                    bulk_load(PK0 + (uint32_t)s * PKB, wsrc + (size_t)kb * PKB, PKB, full);
                    ++issued;
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (!ok) {
                report(a.err, 1u);
                for (long long i = (issued > S ? issued - S : 0); i < issued; ++i)   // let issued copies land first
                    mbar_wait(smem_u32(&bar_full[i % S]), (uint32_t)((i / S) & 1), kWaitBudget);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (even CTA) ----------------
        if (rank == 0) {
            const uint32_t idesc = idesc_i8(2 * kBM, (uint32_t)kPairTileN);
            const uint64_t ad0 = sw128_kmajor_desc(A0), bd0 = sw128_kmajor_desc(B0);
            int s = 0;
            uint32_t ph = 0;
            int j = 0, step = 0;
            for (int tile = pair; tile < a.tiles; tile += npairs, ++j) {
                const int buf = j & 1;
                const uint32_t use = (uint32_t)(j >> 1);
                if (j >= 2) {
                    const bool drained = mbar_wait_cluster(smem_u32(&bar_acc_empty[buf]), (use & 1u) ^ 1u, kWaitBudget);
                    if (!__all_sync(0xFFFFFFFFu, drained)) {
                        ok = false;
                        break;
                    }
                }
                tc_fence_after();
                const uint32_t dcol = tmem + (uint32_t)buf * kPairAccCols;
                for (int kb = 0; kb < kbt; ++kb) {
                    const bool ready = mbar_wait_cluster(smem_u32(&bar_ready[s]), ph, kWaitBudget);
                    if (!__all_sync(0xFFFFFFFFu, ready)) {
                        ok = false;
                        break;
                    }
                    KEA_PTRACE(lane == 0, 3, step);
                    const uint64_t ad = ad0 + (uint64_t)(((uint32_t)s * kPairHalfTile) >> 4);
                    const uint64_t bd = bd0 + (uint64_t)(((uint32_t)s * kPairHalfTile) >> 4);
                    if (elect_one()) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)   // K = 32 per MMA: + 32 bytes = 2 descriptor units
                            mma_i8_pair(dcol, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc,
                                        (kb > 0 || kk > 0) ? 1u : 0u);
                        mma_commit_pair(smem_u32(&bar_empty[s]), (uint16_t)3);
                    }
                    __syncwarp();
                    KEA_PTRACE(lane == 0, 4, step);
                    ++step;
                    if (++s == S) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
                if (!ok) break;
                if (elect_one()) mma_commit_pair(smem_u32(&bar_acc_full[buf]), (uint16_t)3);
                __syncwarp();
            }
            if (!ok && lane == 0) report(a.err, 1u);
            // Every MMA this warp issued completes before the pair tears down its shared and tensor memory.
            if (elect_one()) mma_commit_pair(smem_u32(&bar_drain), (uint16_t)1);
            __syncwarp();
            mbar_wait(smem_u32(&bar_drain), 0u, kWaitBudget);
            __syncwarp();
        }
    } else if (warp >= kPairExpWarp0) {
        // ---------------- expanders ----------------
        // Two groups of four warps take alternate k-blocks, so one group's fence and barrier round trip overlaps the
        // other group's expansion.
        const int eg = (warp - kPairExpWarp0) / kPairExpGroupWarps;             // group
        const int e = threadIdx.x - (kPairExpWarp0 + eg * kPairExpGroupWarps) * 32;   // thread within the group
        const uint32_t ready0 = map_to_rank(smem_u32(&bar_ready[0]), 0u);
        constexpr int units = kPanelN * (WBITS == 1 ? 4 : 8);
        int my_tiles = 0;
        for (int tile = pair; tile < a.tiles; tile += npairs) ++my_tiles;
        const int steps = my_tiles * kbt;
        for (int step = eg; step < steps; step += kPairExpGroups) {
            const int s = step % S;
            const uint32_t ph = (uint32_t)((step / S) & 1);
            const bool landed = mbar_wait(smem_u32(&bar_full[s]), ph, kWaitBudget);
            if (!__all_sync(0xFFFFFFFFu, landed)) {
                ok = false;
                if (lane == 0) report(a.err, 1u);
                break;
            }
            KEA_PTRACE(e == 0, 1, step);
            const uint32_t spk = PK0 + (uint32_t)s * PKB, sb = B0 + (uint32_t)s * kPairHalfTile;
#pragma unroll
            for (int u = e; u < units; u += kPairExpGroupWarps * 32) expand_unit<WBITS>(spk, sb, 7, u);
            fence_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(ready0 + (uint32_t)s * 8u);
            KEA_PTRACE(e == 0, 2, step);
        }
    } else {
        // ---------------- epilogue (warps 2-9) ----------------
        // Warp w reads TMEM lanes 32 (w % 4) .. + 31 (its token rows) and channel half (w - 2) / 4 of every tile;
        // it finishes 32 rows x 64 bytes at a time (32 FP16 or 16 FP32 channels), staged in one of its two 2 KB
        // buffers (64-byte swizzle, as the store's tensor map) and written by one TMA store.
        const int ew = warp - kPairEpiWarp0;
        const int quad = warp & 3, half = ew >> 2;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        const uint32_t stg = STG0 + (uint32_t)ew * 2u * kPairStageOut;
        const uint32_t s_al = STG0 + kPairStagingBytes + (uint32_t)ew * 1024u, s_bi = s_al + 512u;
        const uint32_t acc_empty0 = map_to_rank(smem_u32(&bar_acc_empty[0]), 0u);
        const bool has_bias = a.bias != nullptr;
        int j = 0;
        for (int tile = pair; tile < a.tiles; tile += npairs, ++j) {
            const int buf = j & 1;
            const uint32_t use = (uint32_t)(j >> 1);
            const int mt = tile / a.n_tiles, nt = tile - mt * a.n_tiles;
            const int trow0 = mt * kPairTileM + (int)rank * kBM + quad * 32;
            const int t = trow0 + lane;
            const int nbase = nt * kPairTileN + half * 128;
            // The tile's channel constants do not depend on the MMAs: fetch them while the accumulators fill, one
            // float4 per lane, into the warp's own 1 KB of shared memory (the previous tile's passes are done with it).
            {
                const float4 al = __ldg(reinterpret_cast<const float4 *>(a.alpha + nbase) + lane);
                const float4 bi = has_bias ? __ldg(reinterpret_cast<const float4 *>(a.bias + nbase) + lane)
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
                st_shared_v4(s_al + (uint32_t)lane * 16u, __float_as_uint(al.x), __float_as_uint(al.y),
                             __float_as_uint(al.z), __float_as_uint(al.w));
                st_shared_v4(s_bi + (uint32_t)lane * 16u, __float_as_uint(bi.x), __float_as_uint(bi.y),
                             __float_as_uint(bi.z), __float_as_uint(bi.w));
                __syncwarp();
            }
            const bool done = mbar_wait_sleep(smem_u32(&bar_acc_full[buf]), use & 1u, kWaitBudget, 256);
            if (!__all_sync(0xFFFFFFFFu, done)) {
                ok = false;
                if (lane == 0) report(a.err, 1u);
                break;
            }
            tc_fence_after();
            KEA_PTRACE(ew == 0 && lane == 0, 5, j);
            const float sq = t < a.M ? __ldg(a.qs + t) : 0.f;
            const uint32_t cbase = lane_base + (uint32_t)buf * kPairAccCols + (uint32_t)(half * 128);
            const uint32_t acc_empty = acc_empty0 + (uint32_t)buf * 8u;
            if (a.y_f16) {
                if (has_bias) pair_epilogue_tile<true, true>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq);
                else pair_epilogue_tile<true, false>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq);
            } else {
                if (has_bias) pair_epilogue_tile<false, true>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq);
                else pair_epilogue_tile<false, false>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq);
            }
            KEA_PTRACE(ew == 0 && lane == 0, 6, j);
        }
        // The staging buffers must outlive the stores' reads of them; the global writes complete with the grid.
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
    }

    grid_launch_dependents();
    // Neither CTA of the pair may leave while the other can still arrive on its barriers or the MMAs can still read
    // its shared memory or write its tensor memory.
    tc_fence_before();
    cluster_sync_relaxed_paths();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem, kPairTmemCols);
    }
    KEA_PTRACE(threadIdx.x == 0, 7, 2);
}

}  // namespace kea
