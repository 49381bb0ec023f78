// gemm_pair_kernel.cuh - the large-M low-bit GEMM for sm_100a: a persistent kernel on CTA pairs (tcgen05
// cta_group::2), one or two residual INT8 activation parts.
//
// A pair tile is 256 tokens x 256 channels. The even CTA of a thread-block cluster of two holds tokens 0-127 of the
// tile and channel rows 0-127 (one panel tile); the odd CTA holds tokens 128-255 and channel rows 128-255. Each CTA
// loads its own activation box and packed codes and expands its own half of the weights, so the tensor cores of
// both SMs read only their own shared memory, and every expanded weight serves 256 tokens while each SM stores only
// half of the B operand: per K = 32 step an SM reads 4 KB of activations + 4 KB of weights for 128 x 256 x 32 MACs,
// which keeps shared memory under its bandwidth at the INT8 rate. The even CTA issues tcgen05.mma.cta_group::2
// (M = 256, N = 256) for both; each CTA's tensor memory receives its 128 token rows x 256 channels.
//
// The pairs walk the tile list persistently (pair p takes tiles p, p + pairs, ...). With one part, tensor memory
// holds two 256-column accumulator buffers, so the epilogue of tile i (8 warps per CTA) runs while the MMAs of tile
// i + 1 accumulate into the other buffer. With two parts (P = 2) every load slot holds both parts' activation boxes,
// each expanded weight tile serves both parts' MMAs (one accumulator of 256 columns per part), and the 512 columns
// are one buffer: the next tile's MMAs wait for the epilogue. (A 128-channel tile would keep two buffers, but its
// operand traffic per MAC would take shared memory past its bandwidth.)
//
// Warps per CTA (512 threads):
//   warp 0       producer: per k-block P TMA boxes of activations (128 tokens x 128 k of each part, 128-byte
//                swizzle) and one bulk copy of the packed codes (128 channel rows x 128 k), on this CTA's `full` barrier;
//   warp 1       allocates tensor memory for the pair; in the even CTA one elected lane issues the MMAs, frees each
//                stage in both CTAs (tcgen05.commit to both CTAs' `empty`) and hands finished accumulators to both
//                CTAs' epilogues (`acc_full`);
//   warps 2-7    expanders, two groups of three warps taking alternate k-blocks: packed codes -> INT8 +-1 / -1 0 +1
//                in the 128-byte-swizzled K-major B tile, then arrive on the even CTA's `ready` barrier (6 warp
//                arrivals: the stage is complete in both CTAs);
//   warps 8-15   epilogue: TMEM -> comb_P * alpha (+ bias) (SiLU) -> FP32 / FP16, staged in shared memory and written
//                with TMA stores; then release the buffer (`acc_empty` of the even CTA, 16 warp arrivals).
// Every wait is bounded (kWaitBudget); on expiry the kernel reports KEA_DEVERR_TIMEOUT, lets its copies and MMAs
// drain, and returns.
#pragma once

#include "gemm_kernel.cuh"

namespace kea {

constexpr int kPairWarps = 16;
constexpr int kPairThreads = kPairWarps * 32;     // 512: four warps per SM sub-partition, so 128 registers a thread
constexpr int kPairTileM = 256;                   // tokens per pair tile (128 per CTA)
constexpr int kPairTileN = 256;                   // channels per pair tile (one 128-row panel tile per CTA)
constexpr int kPairExpWarp0 = 2, kPairExpWarps = 6;
constexpr int kPairEpiWarp0 = 8, kPairEpiWarps = 8;
constexpr int kPairExpGroups = 2, kPairExpGroupWarps = kPairExpWarps / kPairExpGroups;
constexpr int kPairMaxStages = 8;                // load slots (activation box + packed codes)
constexpr int kPairBStages = 3;                   // expanded-weight (B) slots
constexpr uint32_t kPairAccCols = 256;            // one accumulator buffer: 128 lanes x 256 INT32 columns
constexpr uint32_t kPairTmemCols = 512;           // two buffers
constexpr uint32_t kPairHalfTile = 16384;         // 128 rows x 128 bytes: one CTA's activation or B tile per stage
constexpr uint32_t kPairStageOut = 2048;          // epilogue staging: one TMA box of 32 rows x 64 bytes, two per warp
constexpr uint32_t kPairStagingBytes = kPairEpiWarps * 2 * kPairStageOut;   // 32 KB
constexpr uint32_t kPairChannelBytes = kPairEpiWarps * 1024;                // alpha + bias of each warp's 128 channels

struct PairArgs {
    const uint8_t *panels;
    const float *qs;             // FP32 [P][m] token scales
    long long qs_stride;         // elements between parts of qs
    const float *alpha;          // FP32 [n]
    const float *bias;           // FP32 [n] or null
    int *acc;                    // optional INT32 [P][m][ld_acc]
    long long ld_acc, acc_stride;
    int M, N, K, kb_total;
    int n_tiles, tiles;          // 256-channel tiles, pair tiles in all
    int m_tiles;                 // 256-token tiles (the weight-stationary kernel's tile order is channel-tile-major)
    int splits, kbs, items;      // K slices per tile, k-blocks per slice, work items = tiles x splits
    int *ws;                     // splits > 1: INT32 partial sums [splits][P][M][N] (scratch), finished by
                                 // splitk_finish_kernel; null otherwise
    int flags;                   // KEA_FLAG_SILU, KEA_FLAG_ORDER1
    const float *res;            // residual FP32 [M][ld_res] (16-byte rows) or null: y = res + res_scale * value
    long long ld_res;
    float res_scale;
    int pdl;
    int y_f16;
    int stages;
    uint32_t *err;
};


// INT32 -> FP32 for |a| < 2^22 (|acc| <= 127 K with K <= 32768 here): exact, so equal to cvt.rn.f32.s32, in two
// full-rate operations. 0x4B400000 is the bit pattern of 1.5 * 2^23, whose mantissa holds a + 2^22 exactly.
KEA_DEVI float int_to_float_exact(int a) { return __fsub_rn(__int_as_float(a + 0x4B400000), 12582912.0f); }

// comb_1, alpha / bias, optional SiLU: one IEEE FP32 rounding per operation (the reference's epilogue order).
template <bool BIAS, bool SILU>
KEA_DEVI float finish1(int acc, float s, float alpha, float bias) {
    const float r = __fmul_rn(int_to_float_exact(acc), s);
    float y = BIAS ? __fmaf_rn(r, alpha, bias) : __fmul_rn(r, alpha);
    if constexpr (SILU) y = silu_approx(y);
    return y;
}

// comb_2 (order 0: fma(a0, s0, a1 * s1); order 1: fma(a1, s1, a0 * s0), the caller passing the parts swapped),
// alpha / bias, optional SiLU: one IEEE FP32 rounding per operation.
template <bool BIAS, bool SILU>
KEA_DEVI float finish2(int lo, int hi, float s_lo, float s_hi, float alpha, float bias) {
    const float r = __fmaf_rn(int_to_float_exact(lo), s_lo, __fmul_rn(int_to_float_exact(hi), s_hi));
    float y = BIAS ? __fmaf_rn(r, alpha, bias) : __fmul_rn(r, alpha);
    if constexpr (SILU) y = silu_approx(y);
    return y;
}

// Work item w: pair tile w % tiles over k-blocks [kb0, kb1) of slice w / tiles (one slice when not split).
KEA_DEVI void pair_item(const PairArgs &a, int w, int &tile, int &slice, int &kb0, int &kb1) {
    tile = w % a.tiles;
    slice = w / a.tiles;
    kb0 = slice * a.kbs;
    kb1 = min(a.kb_total, kb0 + a.kbs);
}

// One epilogue warp's share of a finished tile: its 32 token rows x 128 channels of tensor memory in four chunks of
// 32 columns. The TMEM load of chunk i + 1 is in flight while chunk i is finished in registers (alpha / bias from the
// warp's shared-memory copy). A chunk is 2 KB of FP16 output (one 32 x 64-byte box) or 4 KB of FP32 (two boxes);
// it is staged in the warp's 4 KB buffer (64-byte swizzle, as the store's tensor map) once the store that last used
// that space has read it, then fenced and written by TMA. After the last TMEM load the warp releases the accumulator
// buffer (`acc_empty`, a shared::cluster address).
template <bool F16, bool BIAS, bool SILU>
KEA_DEVI void pair_finish_chunk(uint32_t (&v)[32], uint32_t s_al, uint32_t s_bi, int c, float sq) {
#pragma unroll
    for (int jj = 0; jj < 32; jj += 4) {
        const uint4 alu = ld_shared_v4(s_al + (uint32_t)(c + jj) * 4u);
        uint4 biu = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (BIAS) biu = ld_shared_v4(s_bi + (uint32_t)(c + jj) * 4u);
        const float f0 = finish1<BIAS, SILU>((int)v[jj], sq, __uint_as_float(alu.x), __uint_as_float(biu.x));
        const float f1 = finish1<BIAS, SILU>((int)v[jj + 1], sq, __uint_as_float(alu.y), __uint_as_float(biu.y));
        const float f2 = finish1<BIAS, SILU>((int)v[jj + 2], sq, __uint_as_float(alu.z), __uint_as_float(biu.z));
        const float f3 = finish1<BIAS, SILU>((int)v[jj + 3], sq, __uint_as_float(alu.w), __uint_as_float(biu.w));
        if constexpr (F16) {   // FP16 pairs packed into v[0 .. 16)
            v[jj / 2] = pack_half2(f0, f1);
            v[jj / 2 + 1] = pack_half2(f2, f3);
        } else {               // FP32 bit patterns in place
            v[jj] = __float_as_uint(f0);
            v[jj + 1] = __float_as_uint(f1);
            v[jj + 2] = __float_as_uint(f2);
            v[jj + 3] = __float_as_uint(f3);
        }
    }
}

// comb_2 of one chunk: the order-0 lower part in lo, the other in hi (swapped by the caller for order 1); the
// results replace lo as in pair_finish_chunk.
template <bool F16, bool BIAS, bool SILU>
KEA_DEVI void pair_finish_chunk2(uint32_t (&lo)[32], const uint32_t (&hi)[32], uint32_t s_al, uint32_t s_bi, int c,
                                 float s_lo, float s_hi) {
#pragma unroll
    for (int jj = 0; jj < 32; jj += 4) {
        const uint4 alu = ld_shared_v4(s_al + (uint32_t)(c + jj) * 4u);
        uint4 biu = make_uint4(0u, 0u, 0u, 0u);
        if constexpr (BIAS) biu = ld_shared_v4(s_bi + (uint32_t)(c + jj) * 4u);
        float f[4];
        const float al[4] = {__uint_as_float(alu.x), __uint_as_float(alu.y), __uint_as_float(alu.z), __uint_as_float(alu.w)};
        const float bi[4] = {__uint_as_float(biu.x), __uint_as_float(biu.y), __uint_as_float(biu.z), __uint_as_float(biu.w)};
#pragma unroll
        for (int u = 0; u < 4; ++u) f[u] = finish2<BIAS, SILU>((int)lo[jj + u], (int)hi[jj + u], s_lo, s_hi, al[u], bi[u]);
        if constexpr (F16) {
            lo[jj / 2] = pack_half2(f[0], f[1]);
            lo[jj / 2 + 1] = pack_half2(f[2], f[3]);
        } else {
#pragma unroll
            for (int u = 0; u < 4; ++u) lo[jj + u] = __float_as_uint(f[u]);
        }
    }
}

// residual + scale * value for one chunk of FP32 outputs (bit patterns in v), 32 channels of token row `row`.
KEA_DEVI void pair_add_residual(uint32_t (&v)[32], const float *row, float scale) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
        const float4 r = reinterpret_cast<const float4 *>(row)[q];
        v[4 * q] = __float_as_uint(__fadd_rn(r.x, __fmul_rn(scale, __uint_as_float(v[4 * q]))));
        v[4 * q + 1] = __float_as_uint(__fadd_rn(r.y, __fmul_rn(scale, __uint_as_float(v[4 * q + 1]))));
        v[4 * q + 2] = __float_as_uint(__fadd_rn(r.z, __fmul_rn(scale, __uint_as_float(v[4 * q + 2]))));
        v[4 * q + 3] = __float_as_uint(__fadd_rn(r.w, __fmul_rn(scale, __uint_as_float(v[4 * q + 3]))));
    }
}

template <bool F16>
KEA_DEVI void pair_stage_and_store(const CUtensorMap *ymap, const uint32_t (&v)[32], uint32_t stg, int ci, int n,
                                   int trow0) {
    constexpr int BOXES = F16 ? 1 : 2;     // 64-byte box rows per chunk
    const int lane = threadIdx.x & 31;
    const uint32_t slot = stg + (F16 ? (uint32_t)(ci & 1) * kPairStageOut : 0u);
    if (lane == 0) {   // the store that last read this space must be done with it
        if constexpr (F16) bulk_wait_group_read1();
        else bulk_wait_group_read0();
    }
    __syncwarp();
#pragma unroll
    for (int b = 0; b < BOXES; ++b) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t off = (uint32_t)lane * 64u + (uint32_t)q * 16u;
            const int w0 = b * 16 + q * 4;
            st_shared_v4(slot + (uint32_t)b * kPairStageOut + (off ^ (((off >> 7) & 3u) << 4)), v[w0], v[w0 + 1],
                         v[w0 + 2], v[w0 + 3]);
        }
    }
    fence_async_shared();
    __syncwarp();
    if (lane == 0) {
#pragma unroll
        for (int b = 0; b < BOXES; ++b) tma_store_2d(ymap, slot + (uint32_t)b * kPairStageOut, n + b * 16, trow0);
        bulk_commit_group();
    }
}

KEA_DEVI void pair_load32(uint32_t taddr, uint32_t (&v)[32]) {
    tmem_ld16(taddr, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
    tmem_ld16(taddr + 16u, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
}

template <bool F16, bool BIAS, bool SILU>
KEA_DEVI void pair_epilogue_tile(const PairArgs &a, const CUtensorMap *ymap, uint32_t cbase, uint32_t stg,
                                 uint32_t s_al, uint32_t s_bi, uint32_t acc_empty, int nbase, int trow0, int t, float sq,
                                 int j) {
    const int lane = threadIdx.x & 31;
    const bool tr = threadIdx.x == kPairEpiWarp0 * 32 && j < 16;
    (void)tr;
    uint32_t va[32], vb[32];
    pair_load32(cbase, va);
#pragma unroll
    for (int ci = 0; ci < 4; ci += 2) {
        // chunk ci in va; chunk ci + 1 into vb while va is finished
        tmem_wait_ld();
        tmem_regs_ready(va);
        pair_load32(cbase + (uint32_t)(32 * (ci + 1)), vb);
        if (a.acc && t < a.M) {
            int4 *dst = reinterpret_cast<int4 *>(a.acc + (long long)t * a.ld_acc + nbase + 32 * ci);
#pragma unroll
            for (int q = 0; q < 8; ++q) dst[q] = make_int4((int)va[4 * q], (int)va[4 * q + 1], (int)va[4 * q + 2], (int)va[4 * q + 3]);
        }
        pair_finish_chunk<F16, BIAS, SILU>(va, s_al, s_bi, 32 * ci, sq);
        if constexpr (!F16)
            if (a.res && t < a.M) pair_add_residual(va, a.res + (long long)t * a.ld_res + nbase + 32 * ci, a.res_scale);
        pair_stage_and_store<F16>(ymap, va, stg, ci, nbase + 32 * ci, trow0);
        // chunk ci + 1 in vb; chunk ci + 2 into va
        tmem_wait_ld();
        tmem_regs_ready(vb);
        if (ci + 2 < 4) {
            pair_load32(cbase + (uint32_t)(32 * (ci + 2)), va);
        } else {   // every TMEM read of the buffer is done: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty);
        }
        if (a.acc && t < a.M) {
            int4 *dst = reinterpret_cast<int4 *>(a.acc + (long long)t * a.ld_acc + nbase + 32 * (ci + 1));
#pragma unroll
            for (int q = 0; q < 8; ++q) dst[q] = make_int4((int)vb[4 * q], (int)vb[4 * q + 1], (int)vb[4 * q + 2], (int)vb[4 * q + 3]);
        }
        pair_finish_chunk<F16, BIAS, SILU>(vb, s_al, s_bi, 32 * (ci + 1), sq);
        if constexpr (!F16)
            if (a.res && t < a.M)
                pair_add_residual(vb, a.res + (long long)t * a.ld_res + nbase + 32 * (ci + 1), a.res_scale);
        pair_stage_and_store<F16>(ymap, vb, stg, ci + 1, nbase + 32 * (ci + 1), trow0);
    }
}

// Two parts: per chunk both parts' 32 columns are loaded together (part 1 lies 256 columns on), finished and stored;
// the buffer is released after the last chunk's loads.
template <bool F16, bool BIAS, bool SILU>
KEA_DEVI void pair_epilogue_tile2(const PairArgs &a, const CUtensorMap *ymap, uint32_t cbase, uint32_t stg,
                                  uint32_t s_al, uint32_t s_bi, uint32_t acc_empty, int nbase, int trow0, int t,
                                  float s0, float s1, bool order1) {
    const int lane = threadIdx.x & 31;
    // lo = the part whose product is the fma's first operand (part 0 for order 0, part 1 for order 1)
    const uint32_t col_lo = order1 ? kPairAccCols : 0u, col_hi = order1 ? 0u : kPairAccCols;
    const long long acc_lo = order1 ? a.acc_stride : 0LL, acc_hi = order1 ? 0LL : a.acc_stride;
    const float s_lo = order1 ? s1 : s0, s_hi = order1 ? s0 : s1;
    uint32_t v0[32], v1[32];
#pragma unroll 1
    for (int ci = 0; ci < 4; ++ci) {
        pair_load32(cbase + col_lo + (uint32_t)(32 * ci), v0);
        pair_load32(cbase + col_hi + (uint32_t)(32 * ci), v1);
        tmem_wait_ld();
        tmem_regs_ready(v0);
        tmem_regs_ready(v1);
        if (ci == 3) {   // every TMEM read of the buffer is done: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty);
        }
        if (a.acc && t < a.M) {
            int4 *d0 = reinterpret_cast<int4 *>(a.acc + acc_lo + (long long)t * a.ld_acc + nbase + 32 * ci);
            int4 *d1 = reinterpret_cast<int4 *>(a.acc + acc_hi + (long long)t * a.ld_acc + nbase + 32 * ci);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                d0[q] = make_int4((int)v0[4 * q], (int)v0[4 * q + 1], (int)v0[4 * q + 2], (int)v0[4 * q + 3]);
                d1[q] = make_int4((int)v1[4 * q], (int)v1[4 * q + 1], (int)v1[4 * q + 2], (int)v1[4 * q + 3]);
            }
        }
        pair_finish_chunk2<F16, BIAS, SILU>(v0, v1, s_al, s_bi, 32 * ci, s_lo, s_hi);
        if constexpr (!F16)
            if (a.res && t < a.M) pair_add_residual(v0, a.res + (long long)t * a.ld_res + nbase + 32 * ci, a.res_scale);
        pair_stage_and_store<F16>(ymap, v0, stg, ci, nbase + 32 * ci, trow0);
    }
}

// A K slice's raw INT32 sums of one warp's 32 token rows x 128 channels (every part) into the scratch partials.
template <int P>
KEA_DEVI void pair_partial_tile(const PairArgs &a, uint32_t cbase, uint32_t acc_empty, int nbase, int t, int slice) {
    const int lane = threadIdx.x & 31;
    uint32_t v[P][32];
#pragma unroll 1
    for (int ci = 0; ci < 4; ++ci) {
#pragma unroll
        for (int p = 0; p < P; ++p) pair_load32(cbase + (uint32_t)p * kPairAccCols + (uint32_t)(32 * ci), v[p]);
        tmem_wait_ld();
#pragma unroll
        for (int p = 0; p < P; ++p) tmem_regs_ready(v[p]);
        if (ci == 3) {   // every TMEM read of the buffer is done: hand it back to the MMA warp
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(acc_empty);
        }
        if (t < a.M) {
#pragma unroll
            for (int p = 0; p < P; ++p) {
                int4 *dst = reinterpret_cast<int4 *>(a.ws + (((long long)slice * P + p) * a.M + t) * a.N + nbase +
                                                     32 * ci);
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    dst[q] = make_int4((int)v[p][4 * q], (int)v[p][4 * q + 1], (int)v[p][4 * q + 2], (int)v[p][4 * q + 3]);
            }
        }
    }
}

template <int WBITS, int P>
__global__ void __launch_bounds__(kPairThreads, 1) lowbit_gemm_pair_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                          const __grid_constant__ CUtensorMap ymap,
                                                                          const PairArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t bar_full[kPairMaxStages];    // this CTA's load slot landed (TMA box + codes)
    __shared__ __align__(8) uint64_t bar_empty[kPairMaxStages];   // the pair's MMAs are done with the load slot
    __shared__ __align__(8) uint64_t bar_ready[kPairBStages];     // even CTA: the B slot is expanded in both CTAs
    __shared__ __align__(8) uint64_t bar_bempty[kPairBStages];    // the pair's MMAs are done with the B slot
    __shared__ __align__(8) uint64_t bar_acc_full[2];             // accumulator buffer complete
    __shared__ __align__(8) uint64_t bar_acc_empty[2];            // even CTA: buffer drained by both epilogues
    __shared__ __align__(8) uint64_t bar_drain;                   // even CTA: every issued MMA has completed
    __shared__ uint32_t tmem_slot;

    constexpr uint32_t PKB = (uint32_t)WBITS * kPanelSubBytes;   // packed codes of one CTA per stage
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int pair = (int)(blockIdx.x >> 1), npairs = (int)(gridDim.x >> 1);
    const uint32_t base = (smem_u32(dyn_smem) + 1023u) & ~1023u;
    // Shared memory: [activation boxes: S x P x 16 KB][B tiles: kPairBStages x 16 KB][packed codes: S x PKB][epilogue
    // staging][channel constants]. Load slot s (activations + codes) and B slot b turn over independently: a k-block
    // step i uses load slot i % S and B slot i % kPairBStages, so the loads run S steps ahead of the MMAs while only
    // a few expanded tiles are kept.
    constexpr uint32_t ASLOT = (uint32_t)P * kPairHalfTile;
    constexpr int NBUF = P == 1 ? 2 : 1;   // accumulator buffers
    const int S = a.stages;
    const uint32_t A0 = base, B0 = base + (uint32_t)S * ASLOT;
    const uint32_t PK0 = B0 + (uint32_t)kPairBStages * kPairHalfTile;
    const uint32_t STG0 = (PK0 + (uint32_t)S * PKB + 1023u) & ~1023u;
    const int kbt = a.kb_total;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bar_full[s]), 1);
            mbar_init(smem_u32(&bar_empty[s]), 1);
        }
        for (int b = 0; b < kPairBStages; ++b) {
            mbar_init(smem_u32(&bar_ready[b]), 2 * kPairExpGroupWarps);
            mbar_init(smem_u32(&bar_bempty[b]), 1);
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

    // With programmatic dependent launch, everything below may read what the previous kernel wrote.
    if (a.pdl) grid_dependency_wait();

    bool ok = true;
    if (warp == 0) {
        // ---------------- producer (one lane) ----------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            long long issued = 0;
            const uint32_t tx = ASLOT + PKB;
            for (int w = pair; w < a.items && ok; w += npairs) {
                int tile, slice, kb0, kb1;
                pair_item(a, w, tile, slice, kb0, kb1);
                const int mt = tile / a.n_tiles, nt = tile - mt * a.n_tiles;
                const int t0 = mt * kPairTileM + (int)rank * kBM;
                const uint8_t *wsrc = a.panels + (size_t)(nt * 2 + (int)rank) * (size_t)kbt * PKB;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (issued >= S && !mbar_wait(smem_u32(&bar_empty[s]), ph ^ 1u, kWaitBudget)) {
                        ok = false;
                        break;
                    }
                    const uint32_t full = smem_u32(&bar_full[s]);
                    mbar_arrive_expect_tx(full, tx);
#pragma unroll
                    for (int p = 0; p < P; ++p)   // (k, token, part) boxes
                        tma_load_3d(A0 + (uint32_t)s * ASLOT + (uint32_t)p * kPairHalfTile, &qmap, full, kb * kBK, t0, p);
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
            int j = 0, step = 0;
            for (int w = pair; w < a.items; w += npairs, ++j) {
                int tile, slice, kb0, kb1;
                pair_item(a, w, tile, slice, kb0, kb1);
                const int buf = j % NBUF;
                const uint32_t use = (uint32_t)(j / NBUF);
                if (j >= NBUF) {
                    const bool drained = mbar_wait_cluster(smem_u32(&bar_acc_empty[buf]), (use & 1u) ^ 1u, kWaitBudget);
                    if (!__all_sync(0xFFFFFFFFu, drained)) {
                        ok = false;
                        break;
                    }
                }
                tc_fence_after();
                const uint32_t dcol = tmem + (uint32_t)buf * kPairAccCols;
                for (int kb = kb0; kb < kb1; ++kb, ++step) {
                    const int sa = step % S, sb = step % kPairBStages;
                    const bool ready = mbar_wait_cluster(smem_u32(&bar_ready[sb]), (uint32_t)((step / kPairBStages) & 1),
                                                         kWaitBudget);
                    if (!__all_sync(0xFFFFFFFFu, ready)) {
                        ok = false;
                        break;
                    }
                    const uint64_t ad = ad0 + (uint64_t)(((uint32_t)sa * ASLOT) >> 4);
                    const uint64_t bd = bd0 + (uint64_t)(((uint32_t)sb * kPairHalfTile) >> 4);
                    if (elect_one()) {
#pragma unroll
                        for (int p = 0; p < P; ++p)       // part p: its box, its 256 accumulator columns
#pragma unroll
                            for (int kk = 0; kk < 4; ++kk)   // K = 32 per MMA: + 32 bytes = 2 descriptor units
                                mma_i8_pair(dcol + (uint32_t)p * kPairAccCols,
                                            ad + (uint64_t)((p * kPairHalfTile) >> 4) + (uint64_t)(kk * 2),
                                            bd + (uint64_t)(kk * 2), idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
                        mma_commit_pair(smem_u32(&bar_empty[sa]), (uint16_t)3);
                        mma_commit_pair(smem_u32(&bar_bempty[sb]), (uint16_t)3);
                    }
                    __syncwarp();
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
    } else if (warp < kPairEpiWarp0) {
        // ---------------- expanders ----------------
        // Two groups of three warps take alternate k-blocks, so one group's fence and barrier round trip overlaps the
        // other group's expansion.
        const int eg = (warp - kPairExpWarp0) / kPairExpGroupWarps;             // group
        const int e = threadIdx.x - (kPairExpWarp0 + eg * kPairExpGroupWarps) * 32;   // thread within the group
        const uint32_t ready0 = map_to_rank(smem_u32(&bar_ready[0]), 0u);
        constexpr int units = kPanelN * (WBITS == 1 ? 4 : 8);
        int steps = 0;   // k-blocks of this pair's work items, in order
        for (int w = pair; w < a.items; w += npairs) {
            int tile, slice, kb0, kb1;
            pair_item(a, w, tile, slice, kb0, kb1);
            steps += kb1 - kb0;
        }
        for (int step = eg; step < steps; step += kPairExpGroups) {
            const int sa = step % S, sb = step % kPairBStages;
            // The MMAs that last read B slot sb (step - kPairBStages) are done, then the codes have landed. The order
            // matters: a parity wait on `full` is unambiguous only once the slot's previous fill (step - S) has
            // completed. The MMAs of step - kPairBStages imply every fill up to that step, which covers step - S
            // when S >= kPairBStages; otherwise step - S was this group's own earlier step (S = 2), already waited.
            bool free = true;
            if (step >= kPairBStages)
                free = mbar_wait(smem_u32(&bar_bempty[sb]), (uint32_t)(((step / kPairBStages) & 1) ^ 1), kWaitBudget);
            free = free && mbar_wait(smem_u32(&bar_full[sa]), (uint32_t)((step / S) & 1), kWaitBudget);
            if (!__all_sync(0xFFFFFFFFu, free)) {
                ok = false;
                if (lane == 0) report(a.err, 1u);
                break;
            }
            const uint32_t spk = PK0 + (uint32_t)sa * PKB, sbt = B0 + (uint32_t)sb * kPairHalfTile;
            constexpr int kGroupThreads = kPairExpGroupWarps * 32;
            expand_units<WBITS, (units + kGroupThreads - 1) / kGroupThreads>(spk, sbt, 7, e, kGroupThreads, units);
            fence_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(ready0 + (uint32_t)sb * 8u);
        }
    } else {
        // ---------------- epilogue (warps 8-15) ----------------
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
        for (int w = pair; w < a.items; w += npairs, ++j) {
            const int tile = w % a.tiles;
            const int buf = j % NBUF;
            const uint32_t use = (uint32_t)(j / NBUF);
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
            const float sq = t < a.M ? a.qs[t] : 0.f;
            const float sq1 = (P > 1 && t < a.M) ? a.qs[a.qs_stride + t] : 0.f;
            const uint32_t cbase = lane_base + (uint32_t)buf * kPairAccCols + (uint32_t)(half * 128);
            const uint32_t acc_empty = acc_empty0 + (uint32_t)buf * 8u;
            if (a.splits > 1) {   // a K slice: raw sums to the scratch partials, finished by splitk_finish_kernel
                pair_partial_tile<P>(a, cbase, acc_empty, nbase, t, w / a.tiles);
                continue;
            }
            // one instantiation per (output type, bias, SiLU): no run-time branch inside the finishing loop
            const int variant = (a.y_f16 ? 4 : 0) | (has_bias ? 2 : 0) | (a.flags & 1);
#define KEA_PAIR_EPI(F16, BIAS, SILU)                                                                             \
    if constexpr (P == 1)                                                                                         \
        pair_epilogue_tile<F16, BIAS, SILU>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq, j); \
    else                                                                                                          \
        pair_epilogue_tile2<F16, BIAS, SILU>(a, &ymap, cbase, stg, s_al, s_bi, acc_empty, nbase, trow0, t, sq, sq1, \
                                             (a.flags & 2) != 0)
            switch (variant) {
                case 0: KEA_PAIR_EPI(false, false, false); break;
                case 1: KEA_PAIR_EPI(false, false, true); break;
                case 2: KEA_PAIR_EPI(false, true, false); break;
                case 3: KEA_PAIR_EPI(false, true, true); break;
                case 4: KEA_PAIR_EPI(true, false, false); break;
                case 5: KEA_PAIR_EPI(true, false, true); break;
                case 6: KEA_PAIR_EPI(true, true, false); break;
                default: KEA_PAIR_EPI(true, true, true); break;
            }
#undef KEA_PAIR_EPI
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

// Split-K finish: y[t, n .. n + 3] from the sum over K slices of the pair kernel's INT32 partials
// ws[slice][part][M][N], with the tensor-core kernels' FP32 epilogue (finish_value: comb_P in the order flag's
// order, alpha, bias, SiLU) and optional accumulator / residual outputs, so the result is bit-identical to the
// unsplit pair kernel. One thread per 4 channels of a token; N is a multiple of 256 here.
struct SplitFinishArgs {
    const int *ws;
    int splits, parts, M, N;
    const float *qs;
    long long qs_stride;
    const float *alpha, *bias;
    void *y;
    long long ldy;
    int y_f16;
    int *acc;
    long long ld_acc, acc_stride;
    const float *res;
    long long ld_res;
    float res_scale;
    int flags;
};

__global__ void __launch_bounds__(256) splitk_finish_kernel(const SplitFinishArgs a) {
    grid_dependency_wait();
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;   // (token, 4-channel group)
    const int groups = a.N / 4;
    if (idx >= (long long)a.M * groups) return;
    const int t = (int)(idx / groups), n = (int)(idx - (long long)t * groups) * 4;
    int tot[3][4] = {};
#pragma unroll
    for (int p = 0; p < 3; ++p) {
        if (p >= a.parts) break;
        for (int s = 0; s < a.splits; ++s) {
            const int4 v = *reinterpret_cast<const int4 *>(a.ws + (((long long)s * a.parts + p) * a.M + t) * a.N + n);
            tot[p][0] += v.x;
            tot[p][1] += v.y;
            tot[p][2] += v.z;
            tot[p][3] += v.w;
        }
    }
    float sq[3] = {0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < 3; ++p)
        if (p < a.parts) sq[p] = a.qs[p * a.qs_stride + t];
    const bool has_bias = a.bias != nullptr;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float v = finish_value(tot[0][j], tot[1][j], tot[2][j], sq[0], sq[1], sq[2], a.parts, a.flags,
                               __ldg(a.alpha + n + j), has_bias, has_bias ? __ldg(a.bias + n + j) : 0.f, true);
        if (a.res) v = __fadd_rn(a.res[(long long)t * a.ld_res + n + j], __fmul_rn(a.res_scale, v));
        if (a.y_f16)
            reinterpret_cast<__half *>(a.y)[(long long)t * a.ldy + n + j] = __float2half_rn(v);
        else
            reinterpret_cast<float *>(a.y)[(long long)t * a.ldy + n + j] = v;
    }
    if (a.acc) {
#pragma unroll
        for (int p = 0; p < 3; ++p)
            if (p < a.parts)
#pragma unroll
                for (int j = 0; j < 4; ++j) a.acc[p * a.acc_stride + (long long)t * a.ld_acc + n + j] = tot[p][j];
    }
    grid_launch_dependents();
}

}  // namespace kea
