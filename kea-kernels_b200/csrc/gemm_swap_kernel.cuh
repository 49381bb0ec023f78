// gemm_swap_kernel.cuh - the small-M low-bit GEMM for sm_100a with the operands swapped.
//
// At small M the token count is far below the tcgen05 M = 128 rows, while the channels are many. Here the expanded
// weights are the MMA's A operand (M = 128 channel rows of one panel tile) and the tokens are its B operand: every
// residual part's tokens of one token tile stacked along N (part p's tokens at rows p * mt ..). A CTA computes 128
// channels x all tokens of its tile over its split of K, so each CTA reads only its own K slice of the activations
// (instead of every CTA pulling the whole activation block) and its channels' packed codes exactly once.
//
//   warp 0      producer (one lane): the packed codes of every stage that fits are fetched first (static weights:
//               with programmatic dependent launch this overlaps the previous kernel), then, after
//               griddepcontrol.wait, one TMA box of activations per stage (all parts at once);
//   warp 1      allocates tensor memory; one lane issues tcgen05.mma.kind::i8 (D = 128 channels x rows tokens,
//               INT32 in TMEM, lane = channel, column = stacked token row) and frees each stage with tcgen05.commit;
//   warps 2-9   expand the codes into the 128-byte-swizzled K-major A tile, then run the epilogue: warp w reads TMEM
//               lanes 32 (w % 4) .. + 31, so each thread owns one channel and walks 16-token column chunks; the
//               parts of one token are columns p * mt + t of the same lane, combined in registers.
// The output is written per unit of 32 channels x 16 tokens: the warp finishes the unit's values into a private
// shared-memory tile [16 tokens][32 channels] and one lane stores it with a TMA box store (rows past M and channels
// past N are clipped by the store), so the y rows leave the SM as a few bulk writes instead of per-element stores.
// Split-K: the `splits` CTAs of a thread-block cluster (grid z) share one tile. The 4 x (mt / 16) units are dealt
// round-robin to the ranks; every CTA pushes its INT32 partials of the units it does not own (all parts) into their
// owners' shared memory (which reuses the stage area, once every CTA of the cluster has finished its MMAs), and
// after a cluster barrier each owner adds the received partials to its own (read from tensor memory) and finishes. INT32 sums are exact, so the result
// does not depend on the split.
// Size: 10 warps, at most ~100 KB of shared memory and 128 tensor-memory columns at the Parakeet shapes, so two CTAs
// fit on an SM and the next launch (programmatic dependent launch, triggered at the start) fetches and expands its
// codes while this one finishes.
#pragma once

#include "gemm_kernel.cuh"

namespace kea {

constexpr int kSwapWarps = 10;
constexpr int kSwapThreads = kSwapWarps * 32;   // 320
constexpr int kSwapEpiWarps = 8;                // warps 2-9: expanders, then the epilogue
constexpr int kSwapEpiThreads = kSwapEpiWarps * 32;
constexpr int kSwapStagingBytes = 2 * 16 * 32 * 4;   // per epilogue warp: two [16][32] FP32 unit tiles
constexpr int kSwapMaxRows = 512;          // TMEM columns: every part's tokens of one token tile
constexpr int kSwapMaxTokens = 256;        // tokens per tile (the TMA box's row extent)
constexpr int kSwapStagesMax = 8;
constexpr uint32_t kSwapWTile = 128 * kBK;   // 16 KB: one expanded k-block of 128 channel rows
constexpr int kSwapUnitBytes = 32 * 16 * 4;  // one unit of one part: 32 channels x 16 tokens of INT32

struct SwapArgs {
    const uint8_t *panels;
    const float *qs;
    long long qs_stride;
    const float *alpha;
    const float *bias;
    void *y;
    long long ldy;
    int y_f16;
    int *acc;
    long long ld_acc;
    long long acc_stride;
    const float *res;            // residual FP32 [M][ld_res] or null: y = res + res_scale * value (FP32 y)
    long long ld_res;
    float res_scale;
    int M, N, K;
    int kb_total;
    int splits;                  // K split over a cluster of this many CTAs (grid z)
    int stages;
    int mt;                      // tokens per token tile = TMEM columns per part (a multiple of 16)
    int rows;                    // P * mt: the MMA's N extent
    int nacc;                    // 1, or 4 accumulators (one per K = 32 step) when 4 * rows <= 512
    uint32_t tmem_cols;
    uint32_t a_stage;            // activation bytes of one stage: rows * 128
    uint32_t w_region, pk_region;   // dynamic shared memory offsets of the expanded weights and the packed codes
    uint32_t epi_off;            // the split-K receive buffer, then the epilogue warps' output tiles; 0 (the stage area,
                                 // dead once the MMAs are done) unless they fit only beside the stages
    uint32_t stg_off;            // offset of the output tiles
    int epi_alias;               // 1: the epilogue area overlaps the stage area (split-K: peers must finish first)
    int tma_store;               // 1: y is written with TMA box stores (ymap valid); 0: element stores
    int units_per_owner;         // ceil(4 * mt / 16 / splits)
    int q4d;                     // activations as a 4-D view (k in block, row, part, k-block): one box per stage
    int flags;
    int pdl;
    int stall;                   // test hook: the producer issues no activation copy, so the MMA warp's
                                 // bounded wait runs out and the kernel reports KEA_DEVERR_TIMEOUT
    long long wait_clocks;
    uint32_t *err;
};

// The MMAs of one k128 stage: 4 K = 32 steps; N = rows, split into two MMAs above 256.
template <int NACC>
KEA_DEVI void swap_issue_stage(uint32_t tmem, uint64_t wdesc, uint64_t adesc, uint32_t id0, uint32_t id1, int rows,
                               bool two, bool first) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        const uint32_t accumulate = (!first || (NACC == 1 && kk != 0)) ? 1u : 0u;
        const uint32_t col = NACC > 1 ? (uint32_t)(kk * rows) : 0u;
        mma_i8(tmem + col, wdesc + (uint64_t)(kk * 2), adesc + (uint64_t)(kk * 2), id0, accumulate);
        if (two) mma_i8(tmem + col + 256u, wdesc + (uint64_t)(kk * 2), adesc + (uint64_t)((256 * kBK) >> 4) + (uint64_t)(kk * 2),
                        id1, accumulate);
    }
}

KEA_DEVI void st_shared_u16(uint32_t addr, uint16_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
KEA_DEVI void st_shared_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// comb_P then alpha / bias then optional SiLU, the operations of finish_value with the fast conversion (|acc| < 2^22).
template <int P>
KEA_DEVI float swap_finish_value(uint32_t a0, uint32_t a1, uint32_t a2, float s0, float s1, float s2, int flags,
                                 float alpha, bool has_bias, float bias) {
    float r;
    if (P == 1) {
        r = __fmul_rn(i2f_exact((int)a0), s0);
    } else {
        r = (flags & 2) ? __fmaf_rn(i2f_exact((int)a1), s1, __fmul_rn(i2f_exact((int)a0), s0))
                        : __fmaf_rn(i2f_exact((int)a0), s0, __fmul_rn(i2f_exact((int)a1), s1));
        if (P == 3) r = __fmaf_rn(i2f_exact((int)a2), s2, r);
    }
    r = has_bias ? __fmaf_rn(r, alpha, bias) : __fmul_rn(r, alpha);
    if (flags & 1) r = silu_call(r);
    return r;
}

// Finishes one unit for this lane's channel n: 16 tokens t0 + 16 c + j from the P part accumulators acc[p][j]
// (comb_P, alpha / bias, SiLU, residual), into the warp's output tile [16 tokens][32 channels] at `stg` (TMA-store
// mode) or straight to y; the INT32 accumulators, when asked for, go straight to acc. Requires |acc| < 2^22
// (K <= 32768).
template <int P>
KEA_DEVI void swap_finish_unit(const SwapArgs &a, const uint32_t (&acc)[P][16], int t0, int c, int n, int lane,
                               uint32_t stg, const float *s_qs, float alpha, bool has_bias, float bias) {
    const int tl0 = 16 * c;
    const bool live_n = n < a.N;
    const int flags = a.flags;
    const float *res = a.res;
    const bool f16 = a.y_f16 != 0, tma = a.tma_store != 0;
    if (a.acc && live_n) {
        for (int j = 0; j < 16; ++j) {
            const int t = t0 + tl0 + j;
            if (t >= a.M) break;
#pragma unroll
            for (int p = 0; p < P; ++p) a.acc[p * a.acc_stride + (long long)t * a.ld_acc + n] = (int)acc[p][j];
        }
    }
    float v[16];
#pragma unroll
    for (int g = 0; g < 4; ++g) {   // four tokens at a time: one vector load of each part's token scales
        float sc[P][4];
#pragma unroll
        for (int p = 0; p < P; ++p) {
            const float4 f = *reinterpret_cast<const float4 *>(s_qs + p * a.mt + tl0 + 4 * g);
            sc[p][0] = f.x;
            sc[p][1] = f.y;
            sc[p][2] = f.z;
            sc[p][3] = f.w;
        }
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
            const int j = 4 * g + jj;
            v[j] = swap_finish_value<P>(acc[0][j], P > 1 ? acc[P > 1 ? 1 : 0][j] : 0u, P > 2 ? acc[P > 2 ? 2 : 0][j] : 0u,
                                        sc[0][jj], P > 1 ? sc[P > 1 ? 1 : 0][jj] : 0.f, P > 2 ? sc[P > 2 ? 2 : 0][jj] : 0.f,
                                        flags, alpha, has_bias, bias);
        }
    }
    if (res) {   // the skip connection: residual + scale * value, two roundings, as the unfused expression
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int t = t0 + tl0 + j;
            if (live_n && t < a.M) v[j] = __fadd_rn(res[(long long)t * a.ld_res + n], __fmul_rn(a.res_scale, v[j]));
        }
    }
    if (tma) {
        if (f16) {   // two tokens per conversion instruction, then one 16-bit store each
#pragma unroll
            for (int j = 0; j < 16; j += 2) {
                const __half2 h = __floats2half2_rn(v[j], v[j + 1]);
                const uint32_t w = *reinterpret_cast<const uint32_t *>(&h);
                st_shared_u16(stg + (uint32_t)((j * 32 + lane) * 2), (uint16_t)(w & 0xFFFFu));
                st_shared_u16(stg + (uint32_t)(((j + 1) * 32 + lane) * 2), (uint16_t)(w >> 16));
            }
        } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) st_shared_u32(stg + (uint32_t)((j * 32 + lane) * 4), __float_as_uint(v[j]));
        }
    } else if (live_n) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int t = t0 + tl0 + j;
            if (t >= a.M) break;
            const long long off = (long long)t * a.ldy + n;
            if (f16)
                reinterpret_cast<__half *>(a.y)[off] = __float2half_rn(v[j]);
            else
                reinterpret_cast<float *>(a.y)[off] = v[j];
        }
    }
}

// Stores a finished unit tile: every lane's staging writes, then one lane's TMA box store (32 channels x 16 tokens
// at channel n_base, token t_base); the warp's two tiles alternate, so a tile is rewritten only after the store two
// units back has read it.
KEA_DEVI void swap_store_unit(const CUtensorMap *ymap, uint32_t stg, int n_base, int t_base, int lane) {
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
        tma_store_2d(ymap, stg, n_base, t_base);
        bulk_commit_group();
    }
}

KEA_DEVI void cluster_arrive_relaxed() { asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory"); }

// Waits for the last armed phase of every stage barrier whose copies this thread issued (`issued` copies dealt to
// the stages round-robin), so that no copy is still writing shared memory when the CTA exits.
KEA_DEVI void swap_drain(const uint64_t *bars, int issued, int stages, long long budget) {
    for (int s = 0; s < stages && s < issued; ++s) {
        const int arms = (issued - 1 - s) / stages + 1;
        mbar_wait(smem_u32(&bars[s]), (uint32_t)((arms - 1) & 1), budget);
    }
}


template <int WBITS, int P>
__global__ void __launch_bounds__(kSwapThreads, 2) lowbit_gemm_swap_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                            const __grid_constant__ CUtensorMap ymap,
                                                                            const SwapArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t bar_code[kSwapStagesMax];    // a stage's packed codes landed
    __shared__ __align__(8) uint64_t bar_act[kSwapStagesMax];     // a stage's activation box landed
    __shared__ __align__(8) uint64_t bar_exp[kSwapStagesMax];     // a stage's weights expanded (8 warp arrivals)
    __shared__ __align__(8) uint64_t bar_empty[kSwapStagesMax];   // the stage's MMAs completed
    __shared__ __align__(8) uint64_t bar_acc;                     // every MMA completed
    __shared__ uint32_t tmem_slot;
    __shared__ __align__(16) float s_qs[kSwapMaxRows];
    __shared__ float s_alpha[kBM];
    __shared__ float s_bias[kBM];

    constexpr uint32_t kPkStage = (uint32_t)WBITS * kPanelSubBytes;
    constexpr int kUnits = kBM * (WBITS == 1 ? 4 : 8);          // expansion units of one k-block
    constexpr int kUnitsLog2 = WBITS == 1 ? 9 : 10;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t base = (smem_u32(dyn_smem) + 1023u) & ~1023u;   // 128-byte swizzle atoms need 1024-byte alignment
    const int n0 = blockIdx.x * kPanelN;
    const int t0 = blockIdx.y * a.mt;
    const int rank = a.splits > 1 ? (int)cluster_ctarank() : 0;
    const int kb0 = (int)((long long)a.kb_total * rank / a.splits);
    const int kb1 = (int)((long long)a.kb_total * (rank + 1) / a.splits);
    const int nkb = kb1 - kb0;
    const int S = a.stages;
    const int pre = nkb < S ? nkb : S;          // stages whose codes are fetched before waiting for the previous grid
    const uint32_t A0 = base, W0 = base + a.w_region, PK0 = base + a.pk_region;
    const long long budget = a.wait_clocks;
    const int C = a.mt >> 4;                    // 16-token column chunks per part

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bar_code[s]), 1);
            mbar_init(smem_u32(&bar_act[s]), 1);
            mbar_init(smem_u32(&bar_exp[s]), kSwapEpiWarps);
            mbar_init(smem_u32(&bar_empty[s]), 1);
        }
        mbar_init(smem_u32(&bar_acc), 1);
        fence_barrier_init();
        prefetch_tensormap(&qmap);
        if (a.tma_store) prefetch_tensormap(&ymap);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tmem_slot), a.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    // The next launch may start now: it reads only static weights before its own griddepcontrol.wait, which waits
    // for this grid's completion.
    grid_launch_dependents();
    // Split-K: every CTA of the cluster must be running before a peer stores into its shared memory.
    if (a.splits > 1) cluster_arrive_relaxed();

    int codes_issued = 0, acts_issued = 0;   // producer lane's copies, for the drain at exit
    bool done = true;                        // epilogue warps: the accumulators are complete
    if (warp == 0) {
        // ---------------- producer (one lane issues; the warp reconverges below) ----------------
        if (lane == 0) {
            const uint8_t *wsrc = a.panels + ((size_t)blockIdx.x * (size_t)a.kb_total + (size_t)kb0) * kPkStage;
            for (; codes_issued < pre; ++codes_issued) {
                const uint32_t bar = smem_u32(&bar_code[codes_issued]);
                mbar_arrive_expect_tx(bar, kPkStage);
                bulk_load(PK0 + (uint32_t)codes_issued * kPkStage, wsrc + (size_t)codes_issued * kPkStage, kPkStage, bar);
            }
            if (a.pdl) grid_dependency_wait();
            int s = 0, round = 0;
            for (int i = 0; i < (a.stall ? 0 : nkb); ++i) {
                if (i >= S) {   // the stage's previous MMAs must be done before its codes and activations are replaced
                    if (!mbar_wait(smem_u32(&bar_empty[s]), (uint32_t)((round - 1) & 1), budget)) {
                        report(a.err, 1u);
                        break;
                    }
                    const uint32_t bar = smem_u32(&bar_code[s]);
                    mbar_arrive_expect_tx(bar, kPkStage);
                    bulk_load(PK0 + (uint32_t)s * kPkStage, wsrc + (size_t)i * kPkStage, kPkStage, bar);
                    codes_issued = i + 1;
                }
                const uint32_t abar = smem_u32(&bar_act[s]), dst = A0 + (uint32_t)s * a.a_stage;
                mbar_arrive_expect_tx(abar, a.a_stage);
                if (a.q4d) {
                    tma_load_4d(dst, &qmap, abar, 0, t0, 0, kb0 + i);
                } else {
#pragma unroll
                    for (int p = 0; p < P; ++p)
                        tma_load_3d(dst + (uint32_t)(p * a.mt * kBK), &qmap, abar, (kb0 + i) * kBK, t0, p);
                }
                acts_issued = i + 1;
                if (++s == S) {
                    s = 0;
                    ++round;
                }
            }
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---------------- MMA issuer: the whole warp waits, one elected lane issues ----------------
        const bool two = a.rows > 256;
        const uint32_t id0 = idesc_i8(kBM, (uint32_t)(two ? 256 : a.rows));
        const uint32_t id1 = idesc_i8(kBM, (uint32_t)(two ? a.rows - 256 : 16));
        const uint64_t wd0 = sw128_kmajor_desc(W0), ad0 = sw128_kmajor_desc(A0);
        int s = 0;
        uint32_t ph = 0;
        for (int i = 0; i < nkb; ++i) {
            const bool ready = mbar_wait(smem_u32(&bar_exp[s]), ph, budget) && mbar_wait(smem_u32(&bar_act[s]), ph, budget);
            if (!__all_sync(0xFFFFFFFFu, ready)) {
                if (lane == 0) report(a.err, 1u);
                break;
            }
            // The mbarrier waits order the operands (TMA writes; expander writes behind fence.proxy.async) before
            // the MMAs' shared-memory reads. Fully unrolled stage bodies: no run-time loop around tcgen05.mma.
            const uint64_t wd = wd0 + (uint64_t)(((uint32_t)s * kSwapWTile) >> 4);
            const uint64_t ad = ad0 + (uint64_t)(((uint32_t)s * a.a_stage) >> 4);
            if (elect_one()) {
                if (a.nacc > 1)
                    swap_issue_stage<4>(tmem, wd, ad, id0, id1, a.rows, false, i == 0);
                else
                    swap_issue_stage<1>(tmem, wd, ad, id0, id1, a.rows, two, i == 0);
                mma_commit(smem_u32(&bar_empty[s]));
            }
            __syncwarp();
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }
        if (elect_one()) mma_commit(smem_u32(&bar_acc));   // arrives when every MMA issued above has completed
        __syncwarp();
    } else {
        // ---------------- expanders ----------------
        const int e = threadIdx.x - 64;   // 0 .. 255
        for (int i = e; i < kBM; i += kSwapEpiThreads) {
            const int n = n0 + i;
            s_alpha[i] = n < a.N ? a.alpha[n] : 0.f;
            s_bias[i] = (a.bias && n < a.N) ? a.bias[n] : 0.f;
        }
        bool ok = true;
        // The first `pre` stages' codes were issued together: one pass over all of them behind a single proxy fence,
        // two units per step for instruction-level parallelism.
        bool landed = true;
        for (int s = 0; s < pre; ++s) landed = landed && mbar_wait(smem_u32(&bar_code[s]), 0u, budget);
        if (!__all_sync(0xFFFFFFFFu, landed)) {
            ok = false;
            if (lane == 0) report(a.err, 1u);
        } else {
            const int total = pre << kUnitsLog2;
            for (int f = e; f < total; f += 2 * kSwapEpiThreads) {
                const int f1 = f + kSwapEpiThreads;
                expand_unit<WBITS>(PK0 + (uint32_t)(f >> kUnitsLog2) * kPkStage, W0 + (uint32_t)(f >> kUnitsLog2) * kSwapWTile,
                                   7, f & (kUnits - 1));
                if (f1 < total)
                    expand_unit<WBITS>(PK0 + (uint32_t)(f1 >> kUnitsLog2) * kPkStage,
                                       W0 + (uint32_t)(f1 >> kUnitsLog2) * kSwapWTile, 7, f1 & (kUnits - 1));
            }
            fence_async_shared();
            __syncwarp();
            if (lane == 0)
                for (int s = 0; s < pre; ++s) mbar_arrive(smem_u32(&bar_exp[s]));
        }
        int s = pre < S ? pre : 0;
        uint32_t ph = pre < S ? 0u : 1u;
        for (int i = pre; i < nkb && ok; ++i) {
            if (!__all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&bar_code[s]), ph, budget))) {
                if (lane == 0) report(a.err, 1u);
                break;
            }
            for (int u = e; u < kUnits; u += kSwapEpiThreads)
                expand_unit<WBITS>(PK0 + (uint32_t)s * kPkStage, W0 + (uint32_t)s * kSwapWTile, 7, u);
            fence_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bar_exp[s]));
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }
        // token scales: written by the previous kernel, so read after its completion
        if (a.pdl) grid_dependency_wait();
        for (int i = e; i < P * a.mt; i += kSwapEpiThreads) {
            const int p = i / a.mt, t = t0 + (i - p * a.mt);
            s_qs[i] = t < a.M ? a.qs[p * a.qs_stride + t] : 0.f;
        }
        named_barrier_sync(1, kSwapEpiThreads);   // s_qs / s_alpha / s_bias complete
        done = __all_sync(0xFFFFFFFFu, mbar_wait(smem_u32(&bar_acc), 0u, budget));
        if (!done && lane == 0) report(a.err, 1u);
        tc_fence_after();
    }

    // ---------------- epilogue (warps 2-9) ----------------
    const int quad = warp & 3, sub = (warp - 2) >> 2;   // two warps per TMEM lane quarter, alternate chunks
    const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
    const bool has_bias = a.bias != nullptr;
    const uint32_t stg0 = base + a.stg_off + (uint32_t)((warp - 2) * kSwapStagingBytes);
    int buf = 0;
    if (a.splits == 1) {
        if (warp >= 2 && done) {
            const int ch = quad * 32 + lane;
            const float alpha = s_alpha[ch], bias = s_bias[ch];
            for (int c = sub; c < C; c += 2) {
                uint32_t v[P][16];
#pragma unroll
                for (int p = 0; p < P; ++p) load_acc16(lane_addr, 0, a.nacc, a.rows, p * a.mt + 16 * c, v[p]);
                tmem_wait_ld();
#pragma unroll
                for (int p = 0; p < P; ++p) tmem_regs_ready(v[p]);
                const uint32_t stg = stg0 + (uint32_t)(buf * (kSwapStagingBytes / 2));
                if (a.tma_store) {   // the store that last read this tile (two units back) is done reading it
                    if (lane == 0) bulk_wait_group_read1();
                    __syncwarp();
                }
                swap_finish_unit<P>(a, v, t0, c, n0 + ch, lane, stg, s_qs, alpha, has_bias, bias);
                if (a.tma_store) swap_store_unit(&ymap, stg, n0 + quad * 32, t0 + 16 * c, lane);
                buf ^= 1;
            }
        }
    } else {
        // Every thread of every CTA in the cluster takes the same cluster barriers, in the same order.
        const uint32_t recv = base + a.epi_off;
        const int U = a.units_per_owner;
        cluster_wait();                          // every CTA of the cluster is running
        if (a.epi_alias) cluster_sync_all();     // every CTA's MMAs are done: its stage area may receive partials
        if (warp >= 2) {
            // push: unit u = quad * C + c (this quad's 32 channels x 16 tokens, every part) goes to rank u % splits;
            // the owner keeps its own partial in tensor memory, the others land in its receive slots (one per peer)
            for (int c = sub; c < C; c += 2) {
                const int u = quad * C + c, owner = u % a.splits, lu = u / a.splits;
                if (owner == rank) continue;
                const int slot = rank < owner ? rank : rank - 1;
                uint32_t v[P][16];
                if (done) {
#pragma unroll
                    for (int p = 0; p < P; ++p) load_acc16(lane_addr, 0, a.nacc, a.rows, p * a.mt + 16 * c, v[p]);
                    tmem_wait_ld();
#pragma unroll
                    for (int p = 0; p < P; ++p) tmem_regs_ready(v[p]);
                } else {
#pragma unroll
                    for (int p = 0; p < P; ++p)
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[p][j] = 0u;
                }
                const uint32_t remote = map_to_rank(recv, (uint32_t)owner);
#pragma unroll
                for (int p = 0; p < P; ++p) {
#pragma unroll
                    for (int jq = 0; jq < 4; ++jq)
                        st_cluster_v4(remote + (uint32_t)(((((slot * U + lu) * P + p) * 4 + jq) * 32 + lane) * 16),
                                      v[p][4 * jq], v[p][4 * jq + 1], v[p][4 * jq + 2], v[p][4 * jq + 3]);
                }
            }
        }
        cluster_sync_all();                      // every partial has landed in its owner's shared memory
        if (warp >= 2) {
            // finish the units this rank owns (u = lu * splits + rank): a unit of lane quarter q is taken by one of
            // the two warps that can read q's tensor-memory lanes (its own partial), plus the peers' received slots
            const int units = 4 * C;
            const int own = rank < units ? (units - rank + a.splits - 1) / a.splits : 0;
            int mine = 0;
            for (int lu = 0; lu < own; ++lu) {
                const int u = lu * a.splits + rank;
                const int q = u / C, c = u - q * C;
                if (q != quad || ((mine++) & 1) != sub) continue;
                const int ch = q * 32 + lane;
                uint32_t v[P][16];
                if (done) {
#pragma unroll
                    for (int p = 0; p < P; ++p) load_acc16(lane_addr, 0, a.nacc, a.rows, p * a.mt + 16 * c, v[p]);
                    tmem_wait_ld();
#pragma unroll
                    for (int p = 0; p < P; ++p) tmem_regs_ready(v[p]);
                } else {
#pragma unroll
                    for (int p = 0; p < P; ++p)
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[p][j] = 0u;
                }
                for (int slot = 0; slot + 1 < a.splits; ++slot) {
#pragma unroll
                    for (int p = 0; p < P; ++p) {
#pragma unroll
                        for (int jq = 0; jq < 4; ++jq) {
                            const uint4 x = ld_shared_v4(recv + (uint32_t)(((((slot * U + lu) * P + p) * 4 + jq) * 32 + lane) * 16));
                            v[p][4 * jq] += x.x;
                            v[p][4 * jq + 1] += x.y;
                            v[p][4 * jq + 2] += x.z;
                            v[p][4 * jq + 3] += x.w;
                        }
                    }
                }
                const uint32_t stg = stg0 + (uint32_t)(buf * (kSwapStagingBytes / 2));
                if (a.tma_store) {
                    if (lane == 0) bulk_wait_group_read1();
                    __syncwarp();
                }
                swap_finish_unit<P>(a, v, t0, c, n0 + ch, lane, stg, s_qs, s_alpha[ch], has_bias, s_bias[ch]);
                if (a.tma_store) swap_store_unit(&ymap, stg, n0 + q * 32, t0 + 16 * c, lane);
                buf ^= 1;
            }
        }
    }
    if (warp >= 2 && a.tma_store) {   // the output tiles must outlive the stores' reads of them
        if (lane == 0) bulk_wait_group_read0();
        __syncwarp();
    }

    if (warp == 0 && lane == 0) {   // no copy may still be landing when the CTA exits
        swap_drain(bar_code, codes_issued, S, budget);
        swap_drain(bar_act, acts_issued, S, budget);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, a.tmem_cols);
    }
}

}  // namespace kea
