// gemm_pair_ws_kernel.cuh - the large-M low-bit GEMM for K <= 1024 with the expanded weights resident ("weight
// stationary"), on CTA pairs (tcgen05 cta_group::2), one INT8 activation part.
//
// The pair kernel (gemm_pair_kernel.cuh) re-expands a tile's 256 x K weights every time a pair visits a tile: per
// k128 block each SM's shared memory then carries the TMA activation box (16 KB), the expanded weights (16 KB
// written) and the MMAs' operand reads (its activation box, and its half of the weights for both SMs of the pair:
// 48 KB) - about 80 KB per 4 pair MMAs, past the 128 bytes per clock that keep the MMAs fed (~700 clocks per k-block
// against 545 for the MMAs alone). Here a pair walks a contiguous run of tiles in channel-tile-major order, so it
// keeps one 256-channel tile's weights for several token tiles: each CTA holds its 128 channel rows x all K (<= 8
// k-blocks, 128 KB) expanded in shared memory, re-expanded only when the run reaches the next channel tile, and in
// between only the activation boxes stream in.
//
// Warps per CTA (512 threads), as in the pair kernel:
//   warp 0       producer: per k-block one TMA box of activations (128 tokens x 128 k) into the load ring; when the
//                channel tile changes, first the packed codes of each k-block into a two-slot code ring;
//   warp 1       allocates tensor memory for the pair; in the even CTA one elected lane issues the MMAs (M 256, N 256,
//                K 32) from the activation slot and the resident weights once both CTAs' boxes have landed, frees
//                each activation slot in both CTAs, hands finished accumulators to both epilogues, and when the run
//                leaves a channel tile, frees the weights (`bfree`) once the last MMA that reads them completes; in
//                the odd CTA it forwards each of its landed activation slots to the even CTA (`peer_full`);
//   warps 2-7    expanders, two groups of three warps taking alternate k-blocks (each group owns one code slot): once
//                the previous weights are free, codes -> INT8 in weight slot kb, then arrive on the even CTA's
//                `bready[kb]` (both CTAs' groups);
//   warps 8-15   epilogue of the pair kernel: TMEM -> comb_1 * alpha (+ bias) (SiLU) (+ residual) -> FP32 / FP16,
//                staged and written with TMA stores; two 256-column accumulator buffers.
// Every wait is bounded (kWaitBudget); on expiry the kernel reports KEA_DEVERR_TIMEOUT and returns.
#pragma once

#include "gemm_pair_kernel.cuh"

namespace kea {

constexpr int kWsMaxKb = 8;          // K <= 1024: every k-block's expanded weights stay resident
constexpr int kWsStages = 3;         // activation load slots

// The pair's run of work items: a contiguous share of the tile list (channel-tile-major: tile = nt * m_tiles + mt).
KEA_DEVI void ws_run(const PairArgs &a, int pair, int npairs, int &w0, int &w1) {
    w0 = (int)((long long)a.tiles * pair / npairs);
    w1 = (int)((long long)a.tiles * (pair + 1) / npairs);
}

template <int WBITS>
__global__ void __launch_bounds__(kPairThreads, 1) lowbit_gemm_pair_ws_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                             const __grid_constant__ CUtensorMap ymap,
                                                                             const PairArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t bar_full[kWsStages];     // this CTA's activation slot landed
    __shared__ __align__(8) uint64_t bar_empty[kWsStages];    // the pair's MMAs are done with the activation slot
    __shared__ __align__(8) uint64_t bar_peer_full[kWsStages]; // even CTA: the odd CTA's activation slot landed
    __shared__ __align__(8) uint64_t bar_cfull[2];            // a code slot landed
    __shared__ __align__(8) uint64_t bar_cempty[2];           // the code slot was expanded (one group's 3 warps)
    __shared__ __align__(8) uint64_t bar_bready[kWsMaxKb];    // even CTA: weight slot kb expanded in both CTAs
    __shared__ __align__(8) uint64_t bar_bfree;               // the pair's MMAs are done with the resident weights
    __shared__ __align__(8) uint64_t bar_acc_full[2];         // accumulator buffer complete
    __shared__ __align__(8) uint64_t bar_acc_empty[2];        // even CTA: buffer drained by both epilogues
    __shared__ __align__(8) uint64_t bar_drain;               // even CTA: every issued MMA has completed
    __shared__ uint32_t tmem_slot;

    constexpr uint32_t PKB = (uint32_t)WBITS * kPanelSubBytes;   // packed codes of one CTA per k-block
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
    const uint32_t base = (smem_u32(dyn_smem) + 1023u) & ~1023u;
    const int kbt = a.kb_total;
    // Shared memory: [activation slots: 3 x 16 KB][weights: kbt x 16 KB][code slots: 2 x PKB][epilogue staging]
    // [channel constants].
    const uint32_t A0 = base, B0 = A0 + (uint32_t)kWsStages * kPairHalfTile;
    const uint32_t CK0 = B0 + (uint32_t)kbt * kPairHalfTile;
    const uint32_t STG0 = (CK0 + 2u * PKB + 1023u) & ~1023u;
    int w0, w1;
    ws_run(a, pair, npairs, w0, w1);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kWsStages; ++s) {
            mbar_init(smem_u32(&bar_full[s]), 1);
            mbar_init(smem_u32(&bar_empty[s]), 1);
            mbar_init(smem_u32(&bar_peer_full[s]), 1);
        }
        for (int c = 0; c < 2; ++c) {
            mbar_init(smem_u32(&bar_cfull[c]), 1);
            mbar_init(smem_u32(&bar_cempty[c]), kPairExpGroupWarps);
        }
        for (int kb = 0; kb < kWsMaxKb; ++kb) mbar_init(smem_u32(&bar_bready[kb]), 2 * kPairExpGroupWarps);
        mbar_init(smem_u32(&bar_bfree), 1);
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

    // With programmatic dependent launch, everything below may read what the previous kernel wrote.
    if (a.pdl) grid_dependency_wait();

    bool ok = true;
    if (warp == 0) {
        // ---------------- producer (one lane) ----------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            long long issued = 0;
            int cfills[2] = {0, 0};   // fills of each code slot (slot kb % 2: the expander group of that k-block)
            int prev_nt = -1;
            for (int w = w0; w < w1 && ok; ++w) {
                const int nt = w / a.m_tiles, mt = w - nt * a.m_tiles;
                const bool fresh = nt != prev_nt;
                prev_nt = nt;
                const int t0 = mt * kPairTileM + (int)rank * kBM;
                const uint8_t *wsrc = a.panels + (size_t)(nt * 2 + (int)rank) * (size_t)kbt * PKB;
                for (int kb = 0; kb < kbt; ++kb) {
                    if (fresh) {   // the new channel tile's codes of this k-block, into its group's code slot
                        const int cs = kb & 1;
                        if (cfills[cs] > 0 &&
                            !mbar_wait(smem_u32(&bar_cempty[cs]), (uint32_t)((cfills[cs] - 1) & 1), kWaitBudget)) {
                            ok = false;
                            break;
                        }
                        const uint32_t cf = smem_u32(&bar_cfull[cs]);
                        mbar_arrive_expect_tx(cf, PKB);
                        bulk_load(CK0 + (uint32_t)cs * PKB, wsrc + (size_t)kb * PKB, PKB, cf);
                        ++cfills[cs];
                    }
                    if (issued >= kWsStages && !mbar_wait(smem_u32(&bar_empty[s]), ph ^ 1u, kWaitBudget)) {
                        ok = false;
                        break;
                    }
                    const uint32_t full = smem_u32(&bar_full[s]);
                    mbar_arrive_expect_tx(full, kPairHalfTile);
                    tma_load_3d(A0 + (uint32_t)s * kPairHalfTile, &qmap, full, kb * kBK, t0, 0);
                    ++issued;
                    if (++s == kWsStages) {
                        s = 0;
                        ph ^= 1u;
                    }
                }
            }
            if (!ok) {
                report(a.err, 1u);
                for (long long i = (issued > kWsStages ? issued - kWsStages : 0); i < issued; ++i)   // issued copies land
                    mbar_wait(smem_u32(&bar_full[i % kWsStages]), (uint32_t)((i / kWsStages) & 1), kWaitBudget);
                for (int cs = 0; cs < 2; ++cs)   // the last fill of each code slot
                    if (cfills[cs] > 0) mbar_wait(smem_u32(&bar_cfull[cs]), (uint32_t)((cfills[cs] - 1) & 1), kWaitBudget);
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer (even CTA) ----------------
        if (rank == 0) {
            const uint32_t idesc = idesc_i8(2 * kBM, (uint32_t)kPairTileN);
            const uint64_t ad0 = sw128_kmajor_desc(A0), bd0 = sw128_kmajor_desc(B0);
            int j = 0, step = 0, gen = -1, prev_nt = -1;
            for (int w = w0; w < w1; ++w, ++j) {
                const int nt = w / a.m_tiles;
                const bool fresh = nt != prev_nt;
                prev_nt = nt;
                if (fresh) ++gen;
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
                for (int kb = 0; kb < kbt; ++kb, ++step) {
                    const int sa = step % kWsStages;
                    // the weights (fresh channel tile), this CTA's activation box, and the odd CTA's (forwarded)
                    const uint32_t aph = (uint32_t)((step / kWsStages) & 1);
                    bool ready = !fresh || mbar_wait_cluster(smem_u32(&bar_bready[kb]), (uint32_t)(gen & 1), kWaitBudget);
                    ready = ready && mbar_wait(smem_u32(&bar_full[sa]), aph, kWaitBudget) &&
                            mbar_wait_cluster(smem_u32(&bar_peer_full[sa]), aph, kWaitBudget);
                    if (!__all_sync(0xFFFFFFFFu, ready)) {
                        ok = false;
                        break;
                    }
                    const uint64_t ad = ad0 + (uint64_t)(((uint32_t)sa * kPairHalfTile) >> 4);
                    const uint64_t bd = bd0 + (uint64_t)(((uint32_t)kb * kPairHalfTile) >> 4);
                    if (elect_one()) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk)   // K = 32 per MMA: + 32 bytes = 2 descriptor units
                            mma_i8_pair(dcol, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc,
                                        (kb > 0 || kk > 0) ? 1u : 0u);
                        mma_commit_pair(smem_u32(&bar_empty[sa]), (uint16_t)3);
                    }
                    __syncwarp();
                }
                if (!ok) break;
                if (elect_one()) {
                    mma_commit_pair(smem_u32(&bar_acc_full[buf]), (uint16_t)3);
                    // leaving this channel tile: the weights are free once these MMAs complete
                    if (w + 1 == w1 || (w + 1) / a.m_tiles != nt) mma_commit_pair(smem_u32(&bar_bfree), (uint16_t)3);
                }
                __syncwarp();
            }
            if (!ok && lane == 0) report(a.err, 1u);
            // Every MMA this warp issued completes before the pair tears down its shared and tensor memory.
            if (elect_one()) mma_commit_pair(smem_u32(&bar_drain), (uint16_t)1);
            __syncwarp();
            mbar_wait(smem_u32(&bar_drain), 0u, kWaitBudget);
            __syncwarp();
        } else {
            // The odd CTA's activation boxes feed the even CTA's MMAs: forward each landed slot to the even CTA (its
            // producer may run behind the even one's, e.g. while the code ring refills at a new channel tile).
            const uint32_t peer0 = map_to_rank(smem_u32(&bar_peer_full[0]), 0u);
            int step = 0;
            for (int w = w0; w < w1 && ok; ++w) {
                for (int kb = 0; kb < kbt; ++kb, ++step) {
                    const int sa = step % kWsStages;
                    if (!__all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&bar_full[sa]), (uint32_t)((step / kWsStages) & 1),
                                                           kWaitBudget))) {
                        ok = false;
                        if (lane == 0) report(a.err, 1u);
                        break;
                    }
                    if (lane == 0) mbar_arrive_cluster(peer0 + (uint32_t)sa * 8u);
                    __syncwarp();
                }
            }
        }
    } else if (warp < kPairEpiWarp0) {
        // ---------------- expanders ----------------
        const int eg = (warp - kPairExpWarp0) / kPairExpGroupWarps;             // group: k-blocks kb % 2 == eg
        const int e = threadIdx.x - (kPairExpWarp0 + eg * kPairExpGroupWarps) * 32;   // thread within the group
        const uint32_t bready0 = map_to_rank(smem_u32(&bar_bready[0]), 0u);
        constexpr int units = kPanelN * (WBITS == 1 ? 4 : 8);
        constexpr int kGroupThreads = kPairExpGroupWarps * 32;
        int gen = -1, prev_nt = -1;
        uint32_t use = 0;   // this group's code slot fills consumed
        for (int w = w0; w < w1 && ok; ++w) {
            const int nt = w / a.m_tiles;
            if (nt == prev_nt) continue;   // same channel tile: the resident weights serve it
            prev_nt = nt;
            ++gen;
            // the previous channel tile's MMAs are done reading the weights
            if (gen > 0 && !__all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&bar_bfree), (uint32_t)((gen - 1) & 1), kWaitBudget))) {
                ok = false;
                if (lane == 0) report(a.err, 1u);
                break;
            }
            for (int kb = eg; kb < kbt; kb += 2, ++use) {
                if (!__all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&bar_cfull[eg]), use & 1u, kWaitBudget))) {
                    ok = false;
                    if (lane == 0) report(a.err, 1u);
                    break;
                }
                expand_units<WBITS, (units + kGroupThreads - 1) / kGroupThreads>(CK0 + (uint32_t)eg * PKB,
                                                                                   B0 + (uint32_t)kb * kPairHalfTile, 7, e,
                                                                                   kGroupThreads, units);
                fence_async_shared();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(smem_u32(&bar_cempty[eg]));              // the code slot may be refilled
                    mbar_arrive_cluster(bready0 + (uint32_t)kb * 8u);    // weight slot kb is ready in this CTA
                }
            }
        }
    } else {
        // ---------------- epilogue (warps 8-15): the pair kernel's, over this run's tiles ----------------
        const int ew = warp - kPairEpiWarp0;
        const int quad = warp & 3, half = ew >> 2;
        const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
        const uint32_t stg = STG0 + (uint32_t)ew * 2u * kPairStageOut;
        const uint32_t s_al = STG0 + kPairStagingBytes + (uint32_t)ew * 1024u, s_bi = s_al + 512u;
        const uint32_t acc_empty0 = map_to_rank(smem_u32(&bar_acc_empty[0]), 0u);
        const bool has_bias = a.bias != nullptr;
        int j = 0, prev_nt = -1;
        for (int w = w0; w < w1; ++w, ++j) {
            const int nt = w / a.m_tiles, mt = w - nt * a.m_tiles;
            const int buf = j & 1;
            const uint32_t use = (uint32_t)(j >> 1);
            const int trow0 = mt * kPairTileM + (int)rank * kBM + quad * 32;
            const int t = trow0 + lane;
            const int nbase = nt * kPairTileN + half * 128;
            if (nt != prev_nt) {   // this channel tile's constants (a new tile of the run only)
                prev_nt = nt;
                // the previous tile's epilogue passes are done with the warp's copy (they ran in program order)
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
            const float sq = t < a.M ? a.qs[t] : 0.f;
            const uint32_t cbase = lane_base + (uint32_t)buf * kPairAccCols + (uint32_t)(half * 128);
            const uint32_t acc_empty = acc_empty0 + (uint32_t)buf * 8u;
            const int variant = (a.y_f16 ? 4 : 0) | (has_bias ? 2 : 0) | (a.flags & 1);
            switch (variant) {
                case 0: pair_epilogue_tile<false, false, false>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq, j); break;
                case 1: pair_epilogue_tile<false, false, true>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq, j); break;
                case 2: pair_epilogue_tile<false, true, false>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq, j); break;
                case 3: pair_epilogue_tile<false, true, true>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq, j); break;
                case 4: pair_epilogue_tile<true, false, false>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq, j); break;
                case 5: pair_epilogue_tile<true, false, true>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq, j); break;
                case 6: pair_epilogue_tile<true, true, false>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq, j); break;
                default: pair_epilogue_tile<true, true, true>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq, j); break;
            }
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
}

}  // namespace kea
