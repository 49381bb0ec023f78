// gemm_kernel.cuh - the low-bit GEMM for sm_100a.
//
// One CTA computes `tile_m` tokens (one or two tcgen05 M = 128 blocks) x `tile_n` output channels (32, 64, 128 or
// 256 = the tcgen05 N) over the k128 blocks of its split of K. 18 warps:
//   warp 0      producer: per stage the packed codes of the tile's channels (cp.async.bulk from the panels) and one
//               TMA tile per (token block, activation part): 128 rows x 128 int8, 128-byte swizzle; the copies are
//               spread over the warp's lanes and complete on the stage's `full` mbarrier;
//   warp 1      allocates tensor memory; one lane issues tcgen05.mma.kind::i8 (A = activations, B = expanded
//               weights, INT32 accumulators in TMEM: one tile_n-column block per token block and part) and frees
//               each stage with tcgen05.commit;
//   warps 2-17  expand the packed codes (1 bit -> int8 +-1, 2 bits -> int8 -1/0/+1) into the 128-byte-swizzled
//               K-major B tile, then run the epilogue: warp w reads TMEM lanes 32 (w % 4) .. + 31, so each thread
//               owns one token row; the four warps of a lane quarter share its columns.
// Split-K: the `splits` CTAs of a thread-block cluster share one output tile. Each pushes its INT32 partials of
// channel group g (4 channels) into the shared memory of the rank that owns g (posted distributed-shared-memory
// stores), and after one cluster barrier every rank sums its groups from local shared memory and finishes them.
// INT32 sums are exact, so the result does not depend on the split.
// Epilogue: comb_P, alpha / bias, optional SiLU; FP32 or FP16 rows stored as 16-byte vectors; optional INT32
// accumulators.
#pragma once

#include <cuda_fp16.h>

#include "ptx.cuh"
#include "quant_common.cuh"

namespace kea {

constexpr int kWarps = 18;
constexpr int kThreads = kWarps * 32;    // 576
constexpr int kEpiWarps = 16;            // warps 2-17
constexpr int kEpiThreads = kEpiWarps * 32;
constexpr int kBM = 128;                 // tokens per tcgen05 M block
constexpr int kPanelN = 128;             // channels per panel tile
constexpr int kBK = 128;                 // k per stage: one 128-byte swizzled row of int8
constexpr int kMaxStages = 8;
constexpr int kMaxTileN = 256;
constexpr int kActTileBytes = kBM * kBK;                 // 16 KB per (token block, part)
constexpr int kPanelSubBytes = kPanelN * 16;               // 2 KB per panel sub-block (wbits sub-blocks per k128)
constexpr long long kWaitBudget = 4000000000LL;            // SM clocks (about 2 s) before a wait gives up

__device__ uint32_t g_device_error;  // the library's own error word (KEA_DEVERR_* bits)


struct GemmArgs {
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
    int M, N, K;
    int tile_n, tm_blocks, splits, stages, kb_total;
    int flags;
    int pdl;                     // launched with programmatic dependent launch: wait for the previous grid
    int vec_y, vec_acc;          // 16-byte vector stores allowed (base and row stride aligned)
    uint32_t recv_off;           // split-K receive buffer offset in dynamic shared memory
    int recv_aliases_stages;     // 1: the receive buffer reuses the stage area (peers must finish first)
    int tma_store;               // 1: stage y in shared memory and write it with TMA stores (ymap is valid)
    int store_swizzle;           // ymap's swizzle span in bytes (64 or 128) = one warp's staged row
    uint32_t tmem_cols;
    uint32_t a_stage, b_stage, pk_stage;   // bytes per stage of the activation / expanded-weight / packed regions
    uint32_t b_region, pk_region;         // region offsets in dynamic shared memory (the activation region is at 0)
    int q4d;                     // qmap is 4-D (k in block, row, k-block, part) with 128 * tm_blocks-row boxes
    int oneshot;                 // the whole K range of the CTA arrives at once, in `chunks` pairs of TMA boxes of
                                 // kbox k-blocks each, chunk c on bar_full[c] (expansion and MMAs of chunk 0 overlap
                                 // the landing of chunk 1)
    int chunks;
    int kbox;                    // k-blocks per activation / panel box in one-shot mode
    uint32_t act_tx;             // activation bytes one stage receives (boxes shrink to the rows that exist)
    int nacc;                    // independent accumulators per (token block, part): 1, or 4 for narrow tiles (one per
                                 // K = 32 step, summed in the epilogue) so back-to-back MMAs do not wait on each other
    uint32_t a_stride;           // distance between consecutive stages' activation tiles (one-shot boxes are dense:
                                 // rows * 128 bytes; the MMA's reads past a short tile only reach unstored rows)
    const float *res;            // residual FP32 [M][ld_res] or null: y = res + res_scale * value (FP32 y)
    long long ld_res;
    float res_scale;
    int stack;                   // 1: the P parts are stacked along the rows of one 128-row tile (part p's tokens at
                                 // rows p * mp ..), so one accumulator and one MMA per K step serve every part;
                                 // qmap is then (k, row, part, k-block) with boxes of mp rows x P parts
    int mp;                      // stacked rows per part: M rounded up to the 8-row swizzle atom
    uint32_t *err;
    // Fused prologue quantizer (fq = 1; one-shot, one token tile, one part, K unsplit, K <= 1024): the CTAs of a
    // thread-block cluster of kFqCluster along N quantize the FP32 rows themselves - CTA rank r's epilogue warp w takes
    // token row r + kFqCluster * w - into the cluster's scratch [128][K] INT8 + [128] scales, then a cluster barrier,
    // then the activation boxes are read from that scratch (qmap covers [clusters * 128][K]).
    int fq;
    const float *fq_x;           // row m at fq_x + (m / fq_t) * fq_xb + (m % fq_t) * fq_xt, unit stride along K
    long long fq_xb, fq_xt;
    int fq_t;
    int fq_silu;                 // input SiLU
    const float *fq_nw, *fq_nb;  // LayerNorm (fq_nw null: none), staged in shared memory at fq_off
    float fq_eps;
    const float *fq_pnw, *fq_pnb;   // pre-norm applied first (null: none), staged at fq_off + 2 K floats
    float fq_peps;
    uint32_t fq_off;             // within the activation region (empty until the quantized rows are loaded)
    int8_t *fq_scr;              // [cluster][128][K]
    float *fq_qs_scr;            // [cluster][128]
    int8_t *fq_q;                // optional copies for the caller, written by cluster 0: codes [M][fq_ldq], scales
    float *fq_qs;                // [M], pre-norm output [M][fq_ldn]
    int fq_ldq;
    float *fq_normed;
    long long fq_ldn;
};
constexpr int kFqCluster = 8;

// ---- weight expansion --------------------------------------------------------------------------------------
KEA_DEVI uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}
// Byte tables indexed by a code nibble (prmt selector, low 16 bits = 4 output bytes): 1 bit - 0 -> int8 -1 (0xFF),
// 1 -> +1; 2 bits - 00 -> 0, 01 -> +1, 10 -> -1.
constexpr uint32_t kSignTable = 0x000001FFu;
constexpr uint32_t kTernaryTable = 0x00FF0100u;
KEA_DEVI uint32_t lookup4(uint32_t table, uint32_t sel) { return prmt(table, 0, sel); }

KEA_DEVI void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
KEA_DEVI uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
    return v;
}
KEA_DEVI uint32_t ld_shared_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
KEA_DEVI void st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared::cluster.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// Packed codes of one stage in shared memory: [panel tile][sub-block s][word j][R rows][4 bytes], R = min(tile_n,
// 128) (the panels' own word-major order). Word j of sub-block s of a channel row holds (1 bit) codes 32 j .. + 31,
// (2 bits) codes 64 s + 16 j .. + 15, interleaved by prepare so each code is one nibble of a masked shift of the word.
// Unit u expands channel row r = u % tile_n: 1 bit - word j = u / tile_n (chunks 2 j and 2 j + 1); 2 bits - chunk
// c = u / tile_n (word c % 4 of sub-block c / 4). A chunk is 16 codes = 16 bytes of the B tile, stored at chunk
// position c ^ (r & 7) of row r (128-byte swizzle). tn_log2 = log2(tile_n).
template <int WBITS>
KEA_DEVI uint32_t unit_word_addr(uint32_t pk, int tn_log2, int u) {
    const int r_log2 = tn_log2 < 7 ? tn_log2 : 7;          // R = min(tile_n, 128)
    const int r = u & ((1 << tn_log2) - 1), q = u >> tn_log2;
    const int pt = r >> r_log2, rr = r & ((1 << r_log2) - 1);
    return pk + ((uint32_t)((((pt * (4 * WBITS) + q) << r_log2) | rr)) << 2);
}
template <int WBITS>
KEA_DEVI void expand_word(uint32_t w, uint32_t dst, int tn_log2, int u) {
    const int r = u & ((1 << tn_log2) - 1), q = u >> tn_log2;
    const uint32_t rowbase = dst + (uint32_t)r * 128;
    const uint32_t sw = (uint32_t)(r & 7);
    if constexpr (WBITS == 1) {   // (w >> j) & 0x11111111: codes 8 j .. 8 j + 7, one per nibble
        const uint32_t s0 = w & 0x11111111u, s1 = (w >> 1) & 0x11111111u;
        const uint32_t s2 = (w >> 2) & 0x11111111u, s3 = (w >> 3) & 0x11111111u;
        st_shared_v4(rowbase + (((uint32_t)(2 * q) ^ sw) << 4), lookup4(kSignTable, s0), lookup4(kSignTable, s0 >> 16),
                     lookup4(kSignTable, s1), lookup4(kSignTable, s1 >> 16));
        st_shared_v4(rowbase + (((uint32_t)(2 * q + 1) ^ sw) << 4), lookup4(kSignTable, s2), lookup4(kSignTable, s2 >> 16),
                     lookup4(kSignTable, s3), lookup4(kSignTable, s3 >> 16));
    } else {                      // w & 0x33333333: fields 0-7; (w >> 2) & 0x33333333: fields 8-15
        const uint32_t lo = w & 0x33333333u, hi = (w >> 2) & 0x33333333u;
        st_shared_v4(rowbase + (((uint32_t)q ^ sw) << 4), lookup4(kTernaryTable, lo), lookup4(kTernaryTable, lo >> 16),
                     lookup4(kTernaryTable, hi), lookup4(kTernaryTable, hi >> 16));
    }
}
template <int WBITS>
KEA_DEVI void expand_unit(uint32_t pk, uint32_t dst, int tn_log2, int u) {
    expand_word<WBITS>(ld_shared_u32(unit_word_addr<WBITS>(pk, tn_log2, u)), dst, tn_log2, u);
}
// Units u0, u0 + stride, ... (< units) of one stage, at most MAXU of them: every word is loaded first, then each is
// expanded, so the shared-memory loads and the expansion chains of different units overlap instead of running one
// dependent chain after another.
template <int WBITS, int MAXU>
KEA_DEVI void expand_units(uint32_t pk, uint32_t dst, int tn_log2, int u0, int stride, int units) {
    uint32_t w[MAXU];
#pragma unroll
    for (int i = 0; i < MAXU; ++i) {
        const int u = u0 + i * stride;
        w[i] = u < units ? ld_shared_u32(unit_word_addr<WBITS>(pk, tn_log2, u)) : 0u;
    }
#pragma unroll
    for (int i = 0; i < MAXU; ++i) {
        const int u = u0 + i * stride;
        if (u < units) expand_word<WBITS>(w[i], dst, tn_log2, u);
    }
}

// ---- epilogue ---------------------------------------------------------------------------------------------
// SiLU behind a call: the flag is a run-time value here, and an inlined SiLU would be if-converted into predicated
// ex2 / divide sequences that issue for every output even when the flag is off.
__device__ __noinline__ float silu_call(float y) { return silu_approx(y); }

// INT32 -> FP32 without the conversion unit (which is not full-rate on sm_100): exact for |a| < 2^22, where
// 1.5 * 2^23 + a is a float whose bit pattern is the integer sum, and subtracting 1.5 * 2^23 is exact; so it equals
// cvt.rn.f32.s32. Accumulators stay below 2^22 whenever K <= 32768 (|acc| <= 128 K).
KEA_DEVI float i2f_exact(int a) { return __fsub_rn(__int_as_float(a + 0x4B400000), 12582912.0f); }
KEA_DEVI float acc_to_float(int a, bool small) { return small ? i2f_exact(a) : __int2float_rn(a); }

// comb_P then alpha / bias then optional SiLU, one IEEE FP32 rounding per operation. `small`: every accumulator is
// below 2^22 in magnitude (K <= 32768), so the exact fast conversion applies.
KEA_DEVI float finish_value(int a0, int a1, int a2, float s0, float s1, float s2, int parts, int flags,
                            float alpha, bool has_bias, float bias, bool small) {
    float r;
    if (parts == 1) {
        r = __fmul_rn(acc_to_float(a0, small), s0);
    } else {
        r = (flags & 2) ? __fmaf_rn(acc_to_float(a1, small), s1, __fmul_rn(acc_to_float(a0, small), s0))
                        : __fmaf_rn(acc_to_float(a0, small), s0, __fmul_rn(acc_to_float(a1, small), s1));
        if (parts == 3) r = __fmaf_rn(acc_to_float(a2, small), s2, r);
    }
    r = has_bias ? __fmaf_rn(r, alpha, bias) : __fmul_rn(r, alpha);
    if (flags & 1) r = silu_call(r);
    return r;
}

KEA_DEVI uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Finishes and stores CNT (4 or 16) consecutive channels n .. of token t from acc[p][0..CNT). Channel constants
// come from shared memory (s_alpha / s_bias at tile column c).
template <int P, int CNT>
KEA_DEVI void finish_store(const GemmArgs &a, int t, int n, int c, const int (&acc)[P][CNT], const float (&s)[P],
                           const float *s_alpha, const float *s_bias) {
    const bool has_bias = a.bias != nullptr;
    float v[CNT];
#pragma unroll
    for (int j = 0; j < CNT; ++j)
        v[j] = finish_value(acc[0][j], P > 1 ? acc[P > 1 ? 1 : 0][j] : 0, P > 2 ? acc[P > 2 ? 2 : 0][j] : 0, s[0],
                            P > 1 ? s[P > 1 ? 1 : 0] : 0.f, P > 2 ? s[P > 2 ? 2 : 0] : 0.f, P, a.flags,
                            s_alpha[c + j], has_bias, has_bias ? s_bias[c + j] : 0.f, a.K <= 32768);
    const bool full = n + CNT <= a.N;
    if (a.res) {   // residual + scale * value: the two roundings of the unfused `x + s * y`
        const float *r = a.res + (long long)t * a.ld_res + n;
#pragma unroll
        for (int j = 0; j < CNT; ++j)
            if (full || n + j < a.N) v[j] = __fadd_rn(r[j], __fmul_rn(a.res_scale, v[j]));
    }
    const long long off = (long long)t * a.ldy + n;
    if (a.y_f16) {
        __half *y = reinterpret_cast<__half *>(a.y) + off;
        if (full && a.vec_y) {
            if constexpr (CNT % 8 == 0) {
#pragma unroll
                for (int j = 0; j < CNT; j += 8)
                    *reinterpret_cast<uint4 *>(y + j) = make_uint4(pack_half2(v[j], v[j + 1]), pack_half2(v[j + 2], v[j + 3]),
                                                                  pack_half2(v[j + 4], v[j + 5]), pack_half2(v[j + 6], v[j + 7]));
            } else {
#pragma unroll
                for (int j = 0; j < CNT; j += 4)
                    *reinterpret_cast<uint2 *>(y + j) = make_uint2(pack_half2(v[j], v[j + 1]), pack_half2(v[j + 2], v[j + 3]));
            }
        } else {
#pragma unroll
            for (int j = 0; j < CNT; ++j)
                if (n + j < a.N) y[j] = __float2half_rn(v[j]);
        }
    } else {
        float *y = reinterpret_cast<float *>(a.y) + off;
        if (full && a.vec_y) {
#pragma unroll
            for (int j = 0; j < CNT; j += 4) *reinterpret_cast<float4 *>(y + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
            for (int j = 0; j < CNT; ++j)
                if (n + j < a.N) y[j] = v[j];
        }
    }
    if (a.acc) {
#pragma unroll
        for (int p = 0; p < P; ++p) {
            int *dst = a.acc + p * a.acc_stride + (long long)t * a.ld_acc + n;
            if (full && a.vec_acc) {
#pragma unroll
                for (int j = 0; j < CNT; j += 4)
                    *reinterpret_cast<int4 *>(dst + j) = make_int4(acc[p][j], acc[p][j + 1], acc[p][j + 2], acc[p][j + 3]);
            } else {
#pragma unroll
                for (int j = 0; j < CNT; ++j)
                    if (n + j < a.N) dst[j] = acc[p][j];
            }
        }
    }
}

// 16 columns of accumulator block `blk` (nacc partial accumulators of TN columns each, summed exactly).
KEA_DEVI void load_acc16(uint32_t lane_addr, int blk, int nacc, int TN, int c, uint32_t (&v)[16]) {
    const uint32_t col = (uint32_t)(blk * nacc * TN + c);
    tmem_ld16(lane_addr + col, v);
    if (nacc > 1) {
        uint32_t w1[16], w2[16], w3[16];
        tmem_ld16(lane_addr + col + (uint32_t)TN, w1);
        tmem_ld16(lane_addr + col + (uint32_t)(2 * TN), w2);
        tmem_ld16(lane_addr + col + (uint32_t)(3 * TN), w3);
        tmem_wait_ld();
        tmem_regs_ready(v);
        tmem_regs_ready(w1);
        tmem_regs_ready(w2);
        tmem_regs_ready(w3);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = v[j] + w1[j] + w2[j] + w3[j];
    }
}

// The MMAs of one k128 stage: 4 K = 32 steps x P parts x TMB token blocks, D = 128 tokens x TN channels each.
// Accumulator (token block tb, part p) starts at TMEM column ((tb * P + p) * NACC) * TN; with NACC = 4 each K step
// has its own accumulator (summed in the epilogue) so consecutive narrow MMAs do not wait on one another.
template <int P, int TMB, int NACC>
KEA_DEVI void issue_stage(uint32_t tmem, uint64_t ad_s, uint64_t bd_s, uint32_t idesc, int TN, bool first) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        const uint64_t bd = bd_s + (uint64_t)(kk * 2);      // + kk * 32 bytes (descriptor address unit: 16 bytes)
        const uint32_t accumulate = (!first || (NACC == 1 && kk != 0)) ? 1u : 0u;
#pragma unroll
        for (int p = 0; p < P; ++p) {
#pragma unroll
            for (int tb = 0; tb < TMB; ++tb) {
                const uint64_t ad = ad_s + (uint64_t)(((p * TMB + tb) * kActTileBytes + kk * 32) >> 4);
                const uint32_t col = (uint32_t)(((tb * P + p) * NACC + (NACC > 1 ? kk : 0)) * TN);
                mma_i8(tmem + col, ad, bd, idesc, accumulate);
            }
        }
    }
}

KEA_DEVI void named_barrier_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

KEA_DEVI void report(uint32_t *err, uint32_t bits) { atomicOr(err ? err : &g_device_error, bits); }

// The fused prologue quantizer's row work for one epilogue warp (w = 0 .. 15 of CTA rank r in its cluster): token
// row r + kFqCluster * w of the cluster's 128-row block, quantized with quantize_regs_kernel's arithmetic at 32
// threads per row (pre-norm, LayerNorm, input SiLU, one part) into the cluster's scratch; cluster 0 also writes the
// caller's copies (codes with zeroed padding columns, scales, pre-norm output). `ln` holds the staged parameters:
// norm weight, norm bias, pre-norm weight, pre-norm bias, K floats each.
KEA_DEVI void fused_quantize_rows(const GemmArgs &a, int w, int lane, const float *ln) {
    const int cid = (int)(blockIdx.x / kFqCluster), rank = (int)(blockIdx.x % kFqCluster);
    const int row = rank + kFqCluster * w;
    if (row >= a.M) return;
    const int K = a.K;
    const float4 *src = reinterpret_cast<const float4 *>(a.fq_x + (long long)(row / a.fq_t) * a.fq_xb +
                                                         (long long)(row % a.fq_t) * a.fq_xt);
    float4 v[kRowChunks];
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c) {
        const int i = c * 32 + lane;
        v[c] = 4 * i < K ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const bool first = cid == 0;
    if (a.fq_pnw) {
        warp_layer_norm(v, K, lane, ln + 2 * K, a.fq_pnb ? ln + 3 * K : nullptr, a.fq_peps);
        if (first && a.fq_normed) {
            float4 *dst = reinterpret_cast<float4 *>(a.fq_normed + (long long)row * a.fq_ldn);
#pragma unroll
            for (int c = 0; c < kRowChunks; ++c)
                if (4 * (c * 32 + lane) < K) dst[c * 32 + lane] = v[c];
        }
    }
    if (a.fq_nw) warp_layer_norm(v, K, lane, ln, a.fq_nb ? ln + K : nullptr, a.fq_eps);
    uint32_t words[kRowChunks];
    const float scale = warp_quantize_row(v, K, lane, a.fq_silu != 0, words);
    uint32_t *scr = reinterpret_cast<uint32_t *>(a.fq_scr + ((long long)cid * kBM + row) * K);
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c)
        if (4 * (c * 32 + lane) < K) scr[c * 32 + lane] = words[c];
    if (lane == 0) a.fq_qs_scr[cid * kBM + row] = scale;
    if (first && a.fq_q) {
        uint32_t *q = reinterpret_cast<uint32_t *>(a.fq_q + (long long)row * a.fq_ldq);
#pragma unroll
        for (int c = 0; c < kRowChunks; ++c)
            if (4 * (c * 32 + lane) < K) q[c * 32 + lane] = words[c];
        for (int i = K / 4 + lane; i < a.fq_ldq / 4; i += 32) q[i] = 0u;   // padding columns
        if (lane == 0) a.fq_qs[row] = scale;
    }
}

template <int WBITS, int P>
__global__ void __launch_bounds__(kThreads, 1) lowbit_gemm_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                   const __grid_constant__ CUtensorMap ymap,
                                                                   const __grid_constant__ CUtensorMap wmap, const GemmArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t bar_full[kMaxStages];
    __shared__ __align__(8) uint64_t bar_exp[kMaxStages];
    __shared__ __align__(8) uint64_t bar_empty[kMaxStages];
    __shared__ __align__(8) uint64_t bar_acc;
    __shared__ __align__(8) uint64_t bar_w;      // one-shot with programmatic dependent launch: the packed codes
    __shared__ uint32_t tmem_slot;
    __shared__ float s_qs[3 * 2 * kBM];
    __shared__ float s_alpha[kMaxTileN];
    __shared__ float s_bias[kMaxTileN];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t raw = smem_u32(dyn_smem);
    const uint32_t base = (raw + 1023u) & ~1023u;   // 128-byte swizzle atoms need 1024-byte alignment
    const int TN = a.tile_n, TMB = a.tm_blocks;
    const int tn_log2 = 31 - __clz(TN);
    const int n0 = blockIdx.x * TN, t0 = blockIdx.y * (a.stack ? a.mp : TMB * kBM);
    const int rank = a.splits > 1 ? (int)cluster_ctarank() : 0;
    const int kb0 = (int)((long long)a.kb_total * rank / a.splits);
    const int kb1 = (int)((long long)a.kb_total * (rank + 1) / a.splits);
    const int nkb = kb1 - kb0;
    const int S = a.stages;
    const int R = TN < kPanelN ? TN : kPanelN;             // channel rows taken from one panel tile
    const int ptiles = TN / R;                              // panel tiles per CTA (2 when TN = 256)
    // Shared memory: [activation tiles: S x a_stage][expanded weights: S x b_stage][packed codes: S x pk_stage].
    // Stage s: activation tile of (part p, token block tb) at a(s) + (p * TMB + tb) * 16 KB (a part's token blocks
    // are adjacent, so one 256-row TMA box fills both), B tile at b(s), packed codes at pk(s).
    const uint32_t A0 = base, B0 = base + a.b_region, PK0 = base + a.pk_region;
    const uint32_t tx_bytes = a.act_tx + a.pk_stage;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bar_full[s]), 1);
            mbar_init(smem_u32(&bar_exp[s]), kEpiWarps);
            mbar_init(smem_u32(&bar_empty[s]), 1);
        }
        mbar_init(smem_u32(&bar_acc), 1);
        mbar_init(smem_u32(&bar_w), 1);
        fence_barrier_init();
        prefetch_tensormap(&qmap);
        if (a.tma_store) prefetch_tensormap(&ymap);
        if (a.oneshot) prefetch_tensormap(&wmap);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tmem_slot), a.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    // With programmatic dependent launch, everything below may read what the previous kernel wrote. In one-shot
    // mode the packed codes (static weights) are loaded and expanded first, while the previous kernel finishes:
    // only the producer's activation boxes and the expanders' token-scale loads wait for it.
    const bool early_w = a.oneshot && (a.pdl || a.fq);
    if (a.pdl && !early_w) grid_dependency_wait();

    bool ok = true;
    if (warp == 0) {
        // ---------------- producer: the whole warp waits and issues (the warp stays converged) ----------------
        // Panels: [tile][k-block][sub-block][word][128 rows][4 bytes]; this CTA's rows start at n0 % 128.
        const size_t kblock_bytes = (size_t)WBITS * kPanelSubBytes;
        const size_t tile_bytes = (size_t)a.kb_total * kblock_bytes;
        const uint8_t *wsrc = a.panels + (size_t)(n0 / kPanelN) * tile_bytes + (size_t)(n0 % kPanelN) * 4;
        // CTAs that share token rows start at different k-blocks, so they do not all read the same activation
        // lines at once (INT32 accumulation makes the order free).
        const int rot = nkb > 0 ? (int)(blockIdx.x % (unsigned)nkb) : 0;
        const int pk_copies = R == kPanelN ? ptiles : WBITS * 4;
        const int act_copies = a.q4d ? (a.stack ? 1 : P) : TMB * P;
        const int ncopies = pk_copies + act_copies;   // <= 14
        int issued = 0;
        if (a.oneshot) {
            // Every k-block of this CTA at once: one TMA box of the panels (kbox k-blocks x wbits x 4 word planes
            // of this CTA's R rows) and one 4-D box of activations (128 rows x kbox k-blocks), both on bar_full[0].
            if (lane == 0 && early_w) {   // every chunk's codes on bar_w now; the activations once the previous
                const uint32_t wbar = smem_u32(&bar_w);   // kernel is done
                mbar_arrive_expect_tx(wbar, (uint32_t)(a.chunks * a.kbox) * a.pk_stage);
                for (int c = 0; c < a.chunks; ++c) {
                    const int plane0 = ((n0 / kPanelN) * a.kb_total + kb0 + c * a.kbox) * WBITS * 4;
                    tma_load_2d(PK0 + (uint32_t)(c * a.kbox) * a.pk_stage, &wmap, wbar, (n0 % kPanelN) * 4, plane0);
                }
                grid_dependency_wait();
            }
            __syncwarp();
            if (a.fq) {   // the cluster's epilogue warps have quantized its token rows into the scratch
                cluster_arrive();
                cluster_wait();
            }
            // the activation rows: this token tile's, or the cluster's scratch block
            const int arow = a.fq ? (int)(blockIdx.x / kFqCluster) * kBM : t0;
            if (lane == 0) {
                if (a.fq) fence_proxy_async_global();   // generic-proxy stores of the peers, read by TMA below
                for (int c = 0; c < a.chunks; ++c) {
                    const uint32_t full = smem_u32(&bar_full[c]);
                    const int kbc = kb0 + c * a.kbox;
                    mbar_arrive_expect_tx(full, (uint32_t)a.kbox * (early_w ? a.act_tx : tx_bytes));
                    if (!early_w) {
                        const int plane0 = ((n0 / kPanelN) * a.kb_total + kbc) * WBITS * 4;
                        tma_load_2d(PK0 + (uint32_t)(c * a.kbox) * a.pk_stage, &wmap, full, (n0 % kPanelN) * 4, plane0);
                    }
                    const uint32_t adst = A0 + (uint32_t)(c * a.kbox) * a.a_stride;
                    if (a.stack)
                        tma_load_4d(adst, &qmap, full, 0, arow, 0, kbc);
                    else
                        tma_load_4d(adst, &qmap, full, 0, arow, kbc, 0);
                }
            }
            __syncwarp();
            issued = nkb;
        }
        int s = 0, ph = 0, kbi = rot;   // stage slot, its round parity, k-block offset (incremental: no division)
        for (int i = 0; i < (a.oneshot ? 0 : nkb); ++i) {
            if (i >= S) {
                const bool freed = mbar_wait(smem_u32(&bar_empty[s]), (uint32_t)(ph ^ 1), kWaitBudget);
                if (!__all_sync(0xFFFFFFFFu, freed)) {
                    ok = false;
                    break;
                }
            }
            // One lane arms the stage's barrier; then the stage's copies are spread over the warp's lanes
            // (round-robin across stages): issuing a bulk copy holds its thread for a while, so one issuing
            // lane would starve the tensor cores.
            const uint32_t sa = A0 + (uint32_t)s * a.a_stride, spk = PK0 + (uint32_t)s * a.pk_stage;
            const uint32_t full = smem_u32(&bar_full[s]);
            const int kb = kb0 + kbi;
            if (lane == 0) mbar_arrive_expect_tx(full, tx_bytes);
            __syncwarp();
            const int c = (lane - i * ncopies) & 31;   // this lane's copy index in stage i (valid when < ncopies)
            if (c < ncopies) {
                if (c < pk_copies) {
                    if (R == kPanelN)        // whole sub-blocks of one or two panel tiles
                        bulk_load(spk + c * kblock_bytes, wsrc + c * tile_bytes + (size_t)kb * kblock_bytes,
                                  (uint32_t)kblock_bytes, full);
                    else                     // R rows of one word plane
                        bulk_load(spk + c * R * 4, wsrc + (size_t)kb * kblock_bytes + (size_t)c * kPanelN * 4,
                                  (uint32_t)(R * 4), full);
                } else if (a.stack) {        // one box: mp rows of every part
                    tma_load_4d(sa, &qmap, full, 0, t0, 0, kb);
                } else if (a.q4d) {          // one box of 128 * TMB rows per part
                    const int p = c - pk_copies;
                    tma_load_4d(sa + p * TMB * kActTileBytes, &qmap, full, 0, t0, kb, p);
                } else {                     // one 128-row box per (part, token block)
                    const int blk = c - pk_copies, p = blk / TMB, tb = blk - p * TMB;
                    tma_load_3d(sa + blk * kActTileBytes, &qmap, full, kb * kBK, t0 + tb * kBM, p);
                }
            }
            __syncwarp();
            issued = i + 1;
            if (++kbi == nkb) kbi = 0;
            if (++s == S) {
                s = 0;
                ph ^= 1;
            }
        }
        if (!ok) {
            if (lane == 0) report(a.err, 1u);
            if (a.oneshot) {
                if (early_w) mbar_wait(smem_u32(&bar_w), 0u, kWaitBudget);
                for (int c = 0; c < a.chunks; ++c) mbar_wait(smem_u32(&bar_full[c]), 0u, kWaitBudget);
            } else {
                for (int i = (issued > S ? issued - S : 0); i < issued; ++i)   // let issued copies land first
                    mbar_wait(smem_u32(&bar_full[i % S]), (i / S) & 1, kWaitBudget);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: the whole warp waits, lane 0 issues ----------------
        if (a.fq) {   // the fused quantizer's cluster barrier (every thread of the cluster takes part)
            cluster_arrive();
            cluster_wait();
        }
        const uint32_t idesc = idesc_i8(kBM, (uint32_t)TN);
        const uint64_t a_desc0 = sw128_kmajor_desc(A0), b_desc0 = sw128_kmajor_desc(B0);
        if (a.oneshot && nkb > 0) {
            // Every k-block of a chunk is resident and the expanders arrive on its stage barriers in order after one
            // fence, so the chunk's last stage barrier covers it: one wait per chunk, then its MMAs back to back.
            for (int c = 0; c < a.chunks && ok; ++c) {
                const int i0 = c * a.kbox, i1 = min(nkb, i0 + a.kbox);
                if (i0 >= i1) break;
                const bool ready = mbar_wait(smem_u32(&bar_full[c]), 0u, kWaitBudget) &&
                                   mbar_wait(smem_u32(&bar_exp[i1 - 1]), 0u, kWaitBudget);
                if (!__all_sync(0xFFFFFFFFu, ready)) {
                    ok = false;
                    if (lane == 0) report(a.err, 1u);
                } else if (elect_one()) {
                    for (int i = i0; i < i1; ++i) {
                        const uint64_t ad_s = a_desc0 + (uint64_t)((i * a.a_stride) >> 4);
                        const uint64_t bd_s = b_desc0 + (uint64_t)((i * a.b_stage) >> 4);
                        if (a.stack)
                            issue_stage<1, 1, 4>(tmem, ad_s, bd_s, idesc, TN, i == 0);
                        else
                            issue_stage<P, 1, 4>(tmem, ad_s, bd_s, idesc, TN, i == 0);
                    }
                }
                __syncwarp();
            }
        }
        int s = 0;
        uint32_t ph = 0;
        for (int i = 0; i < (a.oneshot ? 0 : nkb); ++i) {
            const bool ready = mbar_wait(smem_u32(&bar_full[a.oneshot ? 0 : s]), a.oneshot ? 0 : ph, kWaitBudget) &&
                               mbar_wait(smem_u32(&bar_exp[s]), ph, kWaitBudget);
            if (!__all_sync(0xFFFFFFFFu, ready)) {
                ok = false;
                if (lane == 0) report(a.err, 1u);
                break;
            }
            // The mbarrier wait orders the operands (TMA writes, or expander writes behind fence.proxy.async) before
            // the MMAs' shared-memory reads; no tcgen05 fence per stage (it would drain the MMA pipe).
            // The whole warp forms the stage's descriptors (warp-uniform values); one elected lane issues the stage's
            // MMAs from a fully unrolled body (no run-time loop bounds around tcgen05.mma, which slow its issue
            // several-fold).
            const uint64_t ad_s = a_desc0 + (uint64_t)((s * a.a_stride) >> 4);
            const uint64_t bd_s = b_desc0 + (uint64_t)((s * a.b_stage) >> 4);
            if (elect_one()) {
                if (a.stack && a.nacc > 1)
                    issue_stage<1, 1, 4>(tmem, ad_s, bd_s, idesc, TN, i == 0);
                else if (a.stack)
                    issue_stage<1, 1, 1>(tmem, ad_s, bd_s, idesc, TN, i == 0);
                else if (TMB == 2)
                    issue_stage<P, 2, 1>(tmem, ad_s, bd_s, idesc, TN, i == 0);
                else if (a.nacc > 1)
                    issue_stage<P, 1, 4>(tmem, ad_s, bd_s, idesc, TN, i == 0);
                else
                    issue_stage<P, 1, 1>(tmem, ad_s, bd_s, idesc, TN, i == 0);
                mma_commit(smem_u32(&bar_empty[s]));
            }
            __syncwarp();
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }
        if (elect_one()) mma_commit(smem_u32(&bar_acc));
        __syncwarp();
    } else {
        // ---------------- expanders ----------------
        const int e = threadIdx.x - 64;   // 0 .. 511
        if (!early_w) {
            for (int i = e; i < P * TMB * kBM; i += kEpiThreads) {
                const int p = i / (TMB * kBM), t = t0 + (i - p * TMB * kBM);
                s_qs[i] = t < a.M ? a.qs[p * a.qs_stride + t] : 0.f;
            }
        }
        for (int i = e; i < TN; i += kEpiThreads) {
            const int n = n0 + i;
            s_alpha[i] = n < a.N ? a.alpha[n] : 0.f;
            s_bias[i] = (a.bias && n < a.N) ? a.bias[n] : 0.f;
        }
        const int units = TN * (WBITS == 1 ? 4 : 8);
        const int units_log2 = tn_log2 + (WBITS == 1 ? 2 : 3);
        if (a.oneshot && early_w) {
            // The codes of every chunk arrive on bar_w, ahead of the activations: expand them all behind one fence,
            // then wait for the previous kernel and read this tile's token scales.
            const bool landed = mbar_wait(smem_u32(&bar_w), 0u, kWaitBudget);
            if (!__all_sync(0xFFFFFFFFu, landed)) {
                ok = false;
                if (lane == 0) report(a.err, 1u);
            } else {
                for (int f = e; f < (nkb << units_log2); f += kEpiThreads) {
                    const int st = f >> units_log2;
                    expand_unit<WBITS>(PK0 + (uint32_t)st * a.pk_stage, B0 + (uint32_t)st * a.b_stage, tn_log2,
                                       f & (units - 1));
                }
                fence_async_shared();
                __syncwarp();
                if (lane == 0)
                    for (int st = 0; st < nkb; ++st) mbar_arrive(smem_u32(&bar_exp[st]));
            }
            if (a.fq) {
                // the LayerNorms' parameters (static) into shared memory before the wait
                float *ln = reinterpret_cast<float *>(dyn_smem + (base - raw) + a.fq_off);
                for (int i = e; i < a.K; i += kEpiThreads) {
                    ln[i] = a.fq_nw ? a.fq_nw[i] : 0.f;
                    ln[a.K + i] = a.fq_nb ? a.fq_nb[i] : 0.f;
                    ln[2 * a.K + i] = a.fq_pnw ? a.fq_pnw[i] : 0.f;
                    ln[3 * a.K + i] = a.fq_pnb ? a.fq_pnb[i] : 0.f;
                }
                named_barrier_sync(4, kEpiThreads);
                grid_dependency_wait();
                fused_quantize_rows(a, (warp - 2), lane, ln);
                fence_proxy_async_global();
                fence_async_shared();   // the parameters' reads before the activation boxes land over them
                cluster_arrive();
                cluster_wait();
                const float *qs_scr = a.fq_qs_scr + (blockIdx.x / kFqCluster) * kBM;
                for (int i = e; i < kBM; i += kEpiThreads) s_qs[i] = i < a.M ? qs_scr[i] : 0.f;
            } else {
                grid_dependency_wait();
                for (int i = e; i < P * TMB * kBM; i += kEpiThreads) {
                    const int p = i / (TMB * kBM), t = t0 + (i - p * TMB * kBM);
                    s_qs[i] = t < a.M ? a.qs[p * a.qs_stride + t] : 0.f;
                }
            }
        } else if (a.oneshot) {
            // Each chunk's k-blocks are resident at once: spread them over the 512 threads, then one proxy fence and
            // the chunk's stage arrivals (a fence per stage would put its latency into every stage of the MMA chain).
            for (int c = 0; c < a.chunks && ok; ++c) {
                const int i0 = c * a.kbox, i1 = min(nkb, i0 + a.kbox);
                if (i0 >= i1) break;
                const bool landed = mbar_wait(smem_u32(&bar_full[c]), 0u, kWaitBudget);
                if (!__all_sync(0xFFFFFFFFu, landed)) {
                    ok = false;
                    if (lane == 0) report(a.err, 1u);
                } else {
                    for (int f = e + (i0 << units_log2); f < (i1 << units_log2); f += kEpiThreads) {
                        const int st = f >> units_log2;
                        expand_unit<WBITS>(PK0 + (uint32_t)st * a.pk_stage, B0 + (uint32_t)st * a.b_stage, tn_log2,
                                           f & (units - 1));
                    }
                    fence_async_shared();
                    __syncwarp();
                    if (lane == 0)
                        for (int st = i0; st < i1; ++st) mbar_arrive(smem_u32(&bar_exp[st]));
                }
            }
        }
        int s = 0;
        uint32_t ph = 0;
        for (int i = 0; i < (a.oneshot ? 0 : nkb); ++i) {
            const bool landed = mbar_wait(smem_u32(&bar_full[a.oneshot ? 0 : s]), a.oneshot ? 0u : ph, kWaitBudget);
            if (!__all_sync(0xFFFFFFFFu, landed)) {
                ok = false;
                if (lane == 0) report(a.err, 1u);
                break;
            }
            const uint32_t spk = PK0 + (uint32_t)s * a.pk_stage, sb = B0 + (uint32_t)s * a.b_stage;
            for (int u = e; u < units; u += kEpiThreads) expand_unit<WBITS>(spk, sb, tn_log2, u);
            fence_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bar_exp[s]));
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }
    }

    // ---------------- epilogue (warps 2-17) ----------------
    // Warp w may read TMEM lanes 32 (w % 4) .. + 31; the four warps of a lane quarter take 16-column chunks
    // sub, sub + 4, ... of every block.
    const int quad = warp & 3;
    const int sub = (warp - 2) >> 2;
    const int row = quad * 32 + lane;           // token row within a 128-token block
    const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
    const int chunks = TN / 16;
    const uint32_t recv = base + a.recv_off;    // split-K receive buffer
    if (warp < 2 && a.splits > 1 && a.recv_aliases_stages) {   // matches the epilogue warps' early barrier
        cluster_arrive();
        cluster_wait();
    }
    if (warp >= 2) {
        named_barrier_sync(1, kEpiThreads);     // s_qs / s_alpha / s_bias complete
        bool done = ok && mbar_wait(smem_u32(&bar_acc), 0, kWaitBudget);
        done = __all_sync(0xFFFFFFFFu, done);
        if (!done && ok && lane == 0) report(a.err, 1u);
        tc_fence_after();
        if (a.stack && a.splits == 1) {
            // Stacked parts: part p of token t sits in TMEM lane p * mp + t, so the lanes of one token live in
            // different warps. Every row goes to shared memory (the stage area, dead now: all MMAs completed),
            // then each (token, 4-channel group) combines its parts: comb_P, alpha / bias, SiLU, store.
            const uint32_t xs = base;
            const int ld = TN + 4;   // int32 row stride: 16 bytes of padding keep a warp's row stores bank-spread
            if (done) {
                for (int ch = sub; ch < chunks; ch += 4) {
                    uint32_t v[16];
                    load_acc16(lane_addr, 0, a.nacc, TN, ch * 16, v);
                    tmem_wait_ld();
                    tmem_regs_ready(v);
#pragma unroll
                    for (int q = 0; q < 4; ++q)
                        st_shared_v4(xs + (uint32_t)((row * ld + ch * 16 + 4 * q) * 4), v[4 * q], v[4 * q + 1],
                                     v[4 * q + 2], v[4 * q + 3]);
                }
            }
            named_barrier_sync(3, kEpiThreads);
            if (done) {
                const int e = threadIdx.x - 64, g_log2 = tn_log2 - 2;   // TN / 4 groups (a power of two)
                for (int i = e; i < (a.mp << g_log2); i += kEpiThreads) {
                    const int tl = i >> g_log2, g = i & ((1 << g_log2) - 1);
                    const int t = t0 + tl;
                    if (t >= a.M || n0 + 4 * g >= a.N) continue;
                    int accv[P][4];
                    float sc[P];
#pragma unroll
                    for (int p = 0; p < P; ++p) {
                        const uint4 u = ld_shared_v4(xs + (uint32_t)(((p * a.mp + tl) * ld + 4 * g) * 4));
                        accv[p][0] = (int)u.x;
                        accv[p][1] = (int)u.y;
                        accv[p][2] = (int)u.z;
                        accv[p][3] = (int)u.w;
                        sc[p] = s_qs[p * TMB * kBM + tl];
                    }
                    finish_store<P, 4>(a, t, n0 + 4 * g, 4 * g, accv, sc, s_alpha, s_bias);
                }
            }
        } else if (a.splits == 1 && a.tma_store) {
            // Each warp stages its 32 token rows x W = TN / 4 channels of y (64 or 128 bytes a row, swizzled like the
            // store's tensor map) in the free stage area, then one lane stores the box with TMA: a few bulk stores
            // instead of thousands of scattered 16-byte ones.
            if (done) {
                const int W = TN / 4, c_lo = sub * W;
                const uint32_t row_bytes = (uint32_t)a.store_swizzle;             // = W * element size
                const uint32_t sw_mask = row_bytes == 128 ? 7u : 3u;
                const bool has_bias = a.bias != nullptr;
                for (int tb = 0; tb < TMB; ++tb) {
                    const int t = t0 + tb * kBM + row;
                    const uint32_t stg = base + (uint32_t)((tb * kEpiWarps + (warp - 2)) * 32) * row_bytes;
                    float s[P];
#pragma unroll
                    for (int p = 0; p < P; ++p) s[p] = s_qs[p * TMB * kBM + tb * kBM + row];
                    for (int c16 = 0; c16 < W; c16 += 16) {
                        const int c = c_lo + c16;
                        uint32_t v[P][16];
#pragma unroll
                        for (int p = 0; p < P; ++p) load_acc16(lane_addr, tb * P + p, a.nacc, TN, c, v[p]);
                        tmem_wait_ld();
#pragma unroll
                        for (int p = 0; p < P; ++p) tmem_regs_ready(v[p]);
                        float f[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            f[j] = finish_value((int)v[0][j], P > 1 ? (int)v[P > 1 ? 1 : 0][j] : 0,
                                                P > 2 ? (int)v[P > 2 ? 2 : 0][j] : 0, s[0], P > 1 ? s[P > 1 ? 1 : 0] : 0.f,
                                                P > 2 ? s[P > 2 ? 2 : 0] : 0.f, P, a.flags, s_alpha[c + j], has_bias,
                                                has_bias ? s_bias[c + j] : 0.f, a.K <= 32768);
                        // 16 values = 32 bytes (fp16) or 64 bytes (fp32) of this thread's staged row
                        if (a.y_f16) {
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const uint32_t off = (uint32_t)lane * row_bytes + (uint32_t)(c16 * 2 + h * 16);
                                const uint32_t phys = off ^ (((off >> 7) & sw_mask) << 4);
                                st_shared_v4(stg + phys, pack_half2(f[8 * h], f[8 * h + 1]), pack_half2(f[8 * h + 2], f[8 * h + 3]),
                                             pack_half2(f[8 * h + 4], f[8 * h + 5]), pack_half2(f[8 * h + 6], f[8 * h + 7]));
                            }
                        } else {
#pragma unroll
                            for (int h = 0; h < 4; ++h) {
                                const uint32_t off = (uint32_t)lane * row_bytes + (uint32_t)(c16 * 4 + h * 16);
                                const uint32_t phys = off ^ (((off >> 7) & sw_mask) << 4);
                                st_shared_v4(stg + phys, __float_as_uint(f[4 * h]), __float_as_uint(f[4 * h + 1]),
                                             __float_as_uint(f[4 * h + 2]), __float_as_uint(f[4 * h + 3]));
                            }
                        }
                        if (a.acc && t < a.M) {
#pragma unroll
                            for (int p = 0; p < P; ++p)
#pragma unroll
                                for (int j = 0; j < 16; ++j)
                                    if (n0 + c + j < a.N) a.acc[p * a.acc_stride + (long long)t * a.ld_acc + n0 + c + j] = (int)v[p][j];
                        }
                    }
                    fence_async_shared();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_2d(&ymap, stg, n0 + c_lo, t0 + tb * kBM + quad * 32);
                        bulk_commit_group();
                    }
                }
                // The staging area must outlive the stores' reads of it; their global writes complete with the grid
                // (a dependent grid's griddepcontrol.wait sees them), so nothing waits for the writes themselves.
                if (lane == 0) bulk_wait_group_read0();
                __syncwarp();
            }
        } else if (a.splits == 1) {
            if (done) {
                for (int tb = 0; tb < TMB; ++tb) {
                    const int t = t0 + tb * kBM + row;
                    float s[P];
#pragma unroll
                    for (int p = 0; p < P; ++p) s[p] = s_qs[p * TMB * kBM + tb * kBM + row];
                    for (int ch = sub; ch < chunks; ch += 4) {
                        const int c = ch * 16;
                        uint32_t v[P][16];
#pragma unroll
                        for (int p = 0; p < P; ++p) load_acc16(lane_addr, tb * P + p, a.nacc, TN, c, v[p]);
                        tmem_wait_ld();
#pragma unroll
                        for (int p = 0; p < P; ++p) tmem_regs_ready(v[p]);
                        if (t < a.M && n0 + c < a.N) {
                            int accv[P][16];
#pragma unroll
                            for (int p = 0; p < P; ++p)
#pragma unroll
                                for (int j = 0; j < 16; ++j) accv[p][j] = (int)v[p][j];
                            finish_store<P, 16>(a, t, n0 + c, c, accv, s, s_alpha, s_bias);
                        }
                    }
                }
            }
        } else {
            // Push this CTA's INT32 partials to the rank that finishes them: channel group g (4 channels) belongs
            // to rank g / per; its receive buffer holds [source rank][block][group - first group of the owner]
            // [row] x 16 bytes. Remote stores are posted; the cluster barrier below makes them visible.
            const int groups = TN / 4;
            const int per = (groups + a.splits - 1) / a.splits;
            // owner = g / per by a reciprocal (exact for g < 1024, per <= 64): no division per group
            const uint32_t inv_per = (65536u + (uint32_t)per - 1u) / (uint32_t)per;
            const int blocks = a.stack ? 1 : TMB * P;
            if (a.recv_aliases_stages) {   // peers may still be in their main loops: wait until every CTA is done
                cluster_arrive();
                cluster_wait();
            }
            for (int blk = 0; blk < blocks; ++blk) {
                // rows past M (or past the stacked parts) are never read by the owner
                const bool live = a.stack ? (row < P * a.mp && t0 + row % a.mp < a.M) : t0 + (blk / P) * kBM + row < a.M;
                for (int ch = sub; ch < chunks; ch += 4) {
                    uint32_t v[16];
                    if (done) {
                        load_acc16(lane_addr, blk, a.nacc, TN, ch * 16, v);
                        tmem_wait_ld();
                        tmem_regs_ready(v);
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = 0;
                    }
                    if (live) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            const int g = ch * 4 + q;
                            const int owner = (int)(((uint32_t)g * inv_per) >> 16);
                            const uint32_t local =
                                recv + (uint32_t)((((rank * blocks + blk) * per + (g - owner * per)) * kBM + row) * 16);
                            if (owner == rank)
                                st_shared_v4(local, v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                            else
                                st_cluster_v4(map_to_rank(local, (uint32_t)owner), v[4 * q], v[4 * q + 1], v[4 * q + 2],
                                              v[4 * q + 3]);
                        }
                    }
                }
            }
        }
    }

    if (a.splits > 1) {
        cluster_sync_all();  // every partial has landed in its owner's shared memory
        if (warp >= 2 && a.stack) {
            // Stacked parts: sum the splits per stacked row into the first source slot, then combine each token's
            // parts (rows p * mp + t) for this rank's channel groups.
            const int groups = TN / 4;
            const int per = (groups + a.splits - 1) / a.splits;
            const int g_lo = rank * per, g_hi = min(groups, g_lo + per);
            if (row < P * a.mp) {
                for (int g = g_lo + sub; g < g_hi; g += 4) {
                    int4 sum = make_int4(0, 0, 0, 0);
                    for (int src = 0; src < a.splits; ++src) {
                        const uint4 u = ld_shared_v4(recv + (uint32_t)(((src * per + (g - g_lo)) * kBM + row) * 16));
                        sum.x += (int)u.x;
                        sum.y += (int)u.y;
                        sum.z += (int)u.z;
                        sum.w += (int)u.w;
                    }
                    st_shared_v4(recv + (uint32_t)(((g - g_lo) * kBM + row) * 16), (uint32_t)sum.x, (uint32_t)sum.y,
                                 (uint32_t)sum.z, (uint32_t)sum.w);
                }
            }
            named_barrier_sync(3, kEpiThreads);
            const int e = threadIdx.x - 64, own = g_hi - g_lo;
            for (int i = e; i < a.mp * own; i += kEpiThreads) {
                const int tl = i / own, gl = i - tl * own;
                const int t = t0 + tl, g = g_lo + gl;
                if (t >= a.M || n0 + 4 * g >= a.N) continue;
                int accv[P][4];
                float sc[P];
#pragma unroll
                for (int p = 0; p < P; ++p) {
                    const uint4 u = ld_shared_v4(recv + (uint32_t)((gl * kBM + p * a.mp + tl) * 16));
                    accv[p][0] = (int)u.x;
                    accv[p][1] = (int)u.y;
                    accv[p][2] = (int)u.z;
                    accv[p][3] = (int)u.w;
                    sc[p] = s_qs[p * TMB * kBM + tl];
                }
                finish_store<P, 4>(a, t, n0 + 4 * g, 4 * g, accv, sc, s_alpha, s_bias);
            }
        } else if (warp >= 2) {
            const int groups = TN / 4;
            const int per = (groups + a.splits - 1) / a.splits;
            const int blocks = TMB * P;
            const int g_lo = rank * per, g_hi = min(groups, g_lo + per);
            for (int tb = 0; tb < TMB; ++tb) {
                const int t = t0 + tb * kBM + row;
                if (t >= a.M) continue;
                float s[P];
#pragma unroll
                for (int p = 0; p < P; ++p) s[p] = s_qs[p * TMB * kBM + tb * kBM + row];
                for (int g = g_lo + sub; g < g_hi; g += 4) {
                    int accv[P][4];
#pragma unroll
                    for (int p = 0; p < P; ++p) {
                        int4 sum = make_int4(0, 0, 0, 0);
                        for (int src = 0; src < a.splits; ++src) {
                            const uint4 u = ld_shared_v4(
                                recv + (uint32_t)((((src * blocks + tb * P + p) * per + (g - g_lo)) * kBM + row) * 16));
                            sum.x += (int)u.x;
                            sum.y += (int)u.y;
                            sum.z += (int)u.z;
                            sum.w += (int)u.w;
                        }
                        accv[p][0] = sum.x;
                        accv[p][1] = sum.y;
                        accv[p][2] = sum.z;
                        accv[p][3] = sum.w;
                    }
                    if (n0 + 4 * g < a.N) finish_store<P, 4>(a, t, n0 + 4 * g, 4 * g, accv, s, s_alpha, s_bias);
                }
            }
        }
    }

    grid_launch_dependents();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, a.tmem_cols);
    }
}

}  // namespace kea
