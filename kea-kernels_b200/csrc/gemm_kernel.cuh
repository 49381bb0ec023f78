// gemm_kernel.cuh - the low-bit GEMM for sm_100a.
//
// One CTA computes a tile of `tile_m` tokens (1 or 2 tcgen05 M=128 blocks) x `tile_n` output channels (128 or 256,
// the tcgen05 N) over the k128 blocks of its split of K:
//   warp 0     producer: per stage one cp.async.bulk per 128-channel panel tile (wbits x 2 KB of packed codes) and
//              one TMA tile per (token block, activation part) (128 rows x 128 int8, 128-byte swizzle), all
//              completing on the stage's `full` mbarrier;
//   warp 1     allocates tensor memory; one thread issues tcgen05.mma.kind::i8 (M = 128 tokens, N = tile_n
//              channels, K = 32) with A = activations and B = expanded weights, INT32 accumulators in TMEM (one
//              tile_n-column block per token block and part), and frees each stage with tcgen05.commit;
//   warps 2-9  expand the packed codes (1 bit -> int8 +-1, 2 bits -> int8 -1/0/+1) into the 128-byte-swizzled
//              K-major B tile, then run the epilogue: each thread owns one token row of a TMEM lane quarter.
// Split-K: the `splits` CTAs of a thread-block cluster share one output tile; each copies its INT32 partials from
// TMEM into its own shared memory, and after a cluster barrier every CTA sums a slice of the channels across the
// cluster through distributed shared memory (exact INT32, so the order does not matter) and finishes it.
// Epilogue: comb_P, alpha / bias, optional SiLU; FP32 or FP16 rows stored as 16-byte vectors; optional INT32
// accumulators.
#pragma once

#include <cuda_fp16.h>

#include "ptx.cuh"

namespace kea {

constexpr int kThreads = 320;            // 10 warps
constexpr int kEpiThreads = 256;         // warps 2-9
constexpr int kBM = 128;                 // tokens per tcgen05 M block
constexpr int kPanelN = 128;             // channels per panel tile
constexpr int kBK = 128;                 // k per stage: one 128-byte swizzled row of int8
constexpr int kMaxStages = 8;
constexpr int kMaxTileN = 256;
constexpr int kActTileBytes = kBM * kBK;                 // 16 KB per (token block, part)
constexpr int kPanelRowBytes = 16;
constexpr int kPanelSubBytes = kPanelN * kPanelRowBytes;   // 2 KB per sub-block (wbits sub-blocks per k128)
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
    int parts, tile_n, tm_blocks, splits, stages, kb_total;
    int flags;
    int vec_y, vec_acc;          // 16-byte vector stores allowed (base and row stride aligned)
    uint32_t tmem_cols;
    uint32_t stage_bytes;
    uint32_t *err;
};

// ---- weight expansion --------------------------------------------------------------------------------------
// `rep` holds one packed byte in all four byte lanes; `mask` selects a single bit per lane. Returns 1 in
// every byte lane whose selected bit is set, else 0 (each lane stays below 0x100, so no carries).
KEA_DEVI uint32_t lane_bits(uint32_t rep, uint32_t mask) { return (((rep & mask) + 0x7F7F7F7Fu) >> 7) & 0x01010101u; }
// 1-bit codes: 1 -> int8 +1 (0x01), 0 -> int8 -1 (0xFF).
KEA_DEVI uint32_t sign_lanes(uint32_t ones) { return ones | ((ones ^ 0x01010101u) * 0xFFu); }
// 2-bit codes: 01 -> +1, 10 -> -1, 00 -> 0 for the four fields of `rep`'s byte.
KEA_DEVI uint32_t ternary_lanes(uint32_t rep) {
    return lane_bits(rep, 0x40100401u) | (lane_bits(rep, 0x80200802u) * 0xFFu);
}
KEA_DEVI uint32_t byte_in_all_lanes(uint32_t word, uint32_t i) { return __byte_perm(word, 0, i * 0x1111u); }

KEA_DEVI void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
KEA_DEVI uint4 ld_shared_v4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
    return v;
}
KEA_DEVI uint2 ld_shared_v2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
    return v;
}
KEA_DEVI int4 ld_cluster_v4(uint32_t addr) {
    int4 v;
    asm volatile("ld.shared::cluster.v4.s32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// Expands chunks [c0, c0 + NCH) (16 codes each) of channel row `row` of one k128 stage. Packed codes of row r of
// a 128-channel panel tile: sub-block s at pk + s * 2048 + (r % 128) * 16, where pk is the tile's packed area.
// Output: the int8 B tile at `dst`, row r at r * 128, 16-byte chunk c stored at chunk c ^ (r & 7).
template <int WBITS, int NCH>
KEA_DEVI void expand_chunks(uint32_t pk, uint32_t dst, int row, int c0) {
    const uint32_t rowbase = dst + row * 128;
    const uint32_t sw = row & 7;
    if constexpr (WBITS == 1) {
        // chunks c0..c0+NCH-1 are packed bytes 2 c0 .. 2 (c0 + NCH) - 1 (LSB first)
        uint32_t w[NCH / 2];
        if constexpr (NCH == 8) {
            const uint4 v = ld_shared_v4(pk + row * kPanelRowBytes);
            w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
        } else {
            const uint2 v = ld_shared_v2(pk + row * kPanelRowBytes + 2 * c0);
            w[0] = v.x; w[1] = v.y;
        }
#pragma unroll
        for (int i = 0; i < NCH; ++i) {
            const uint32_t word = w[i >> 1];
            const uint32_t r0 = byte_in_all_lanes(word, 2 * (i & 1)), r1 = byte_in_all_lanes(word, 2 * (i & 1) + 1);
            st_shared_v4(rowbase + (((c0 + i) ^ sw) << 4), sign_lanes(lane_bits(r0, 0x08040201u)),
                         sign_lanes(lane_bits(r0, 0x80402010u)), sign_lanes(lane_bits(r1, 0x08040201u)),
                         sign_lanes(lane_bits(r1, 0x80402010u)));
        }
    } else {
        // chunk c: sub-block c / 4 (64 codes), packed word c % 4 of it (4 codes per byte)
#pragma unroll
        for (int h = 0; h < NCH / 4; ++h) {
            const int sub = c0 / 4 + h;
            const uint4 v = ld_shared_v4(pk + sub * kPanelSubBytes + row * kPanelRowBytes);
            const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                st_shared_v4(rowbase + (((sub * 4 + i) ^ sw) << 4), ternary_lanes(byte_in_all_lanes(w[i], 0)),
                             ternary_lanes(byte_in_all_lanes(w[i], 1)), ternary_lanes(byte_in_all_lanes(w[i], 2)),
                             ternary_lanes(byte_in_all_lanes(w[i], 3)));
            }
        }
    }
}

// ---- epilogue ---------------------------------------------------------------------------------------------
// comb_P then alpha / bias then optional SiLU, one IEEE FP32 rounding per operation.
KEA_DEVI float finish_value(int a0, int a1, int a2, float s0, float s1, float s2, int parts, int flags,
                            float alpha, bool has_bias, float bias) {
    float r;
    if (parts == 1) {
        r = __fmul_rn(__int2float_rn(a0), s0);
    } else {
        r = (flags & 2) ? __fmaf_rn(__int2float_rn(a1), s1, __fmul_rn(__int2float_rn(a0), s0))
                        : __fmaf_rn(__int2float_rn(a0), s0, __fmul_rn(__int2float_rn(a1), s1));
        if (parts == 3) r = __fmaf_rn(__int2float_rn(a2), s2, r);
    }
    r = has_bias ? __fmaf_rn(r, alpha, bias) : __fmul_rn(r, alpha);
    if (flags & 1) r = silu_approx(r);
    return r;
}

KEA_DEVI uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// Finishes and stores `cnt` (a multiple of 4, <= 16) consecutive channels n .. of token t from acc[p][0..cnt).
// Channel-indexed constants come from shared memory (s_alpha / s_bias at tile column c).
template <int P, int CNT>
KEA_DEVI void finish_store(const GemmArgs &a, int t, int n, int c, const int (&acc)[P][CNT], const float (&s)[P],
                           const float *s_alpha, const float *s_bias) {
    const bool has_bias = a.bias != nullptr;
    float v[CNT];
#pragma unroll
    for (int j = 0; j < CNT; ++j)
        v[j] = finish_value(acc[0][j], P > 1 ? acc[P > 1 ? 1 : 0][j] : 0, P > 2 ? acc[P > 2 ? 2 : 0][j] : 0, s[0],
                            P > 1 ? s[P > 1 ? 1 : 0] : 0.f, P > 2 ? s[P > 2 ? 2 : 0] : 0.f, P, a.flags,
                            s_alpha[c + j], has_bias, has_bias ? s_bias[c + j] : 0.f);
    const long long off = (long long)t * a.ldy + n;
    const bool full = n + CNT <= a.N;
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

KEA_DEVI void named_barrier_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

KEA_DEVI void report(uint32_t *err, uint32_t bits) { atomicOr(err ? err : &g_device_error, bits); }

template <int WBITS, int P>
__global__ void __launch_bounds__(kThreads, 1) lowbit_gemm_kernel(const __grid_constant__ CUtensorMap qmap, const GemmArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t bar_full[kMaxStages];
    __shared__ __align__(8) uint64_t bar_exp[kMaxStages];
    __shared__ __align__(8) uint64_t bar_empty[kMaxStages];
    __shared__ __align__(8) uint64_t bar_acc;
    __shared__ uint32_t tmem_slot;
    __shared__ float s_qs[3 * 2 * kBM];
    __shared__ float s_alpha[kMaxTileN];
    __shared__ float s_bias[kMaxTileN];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t raw = smem_u32(dyn_smem);
    const uint32_t base = (raw + 1023u) & ~1023u;   // 128-byte swizzle atoms need 1024-byte alignment
    const int TN = a.tile_n, TMB = a.tm_blocks;
    const int n0 = blockIdx.x * TN, t0 = blockIdx.y * (TMB * kBM);
    const int rank = a.splits > 1 ? (int)cluster_ctarank() : 0;
    const int kb0 = (int)((long long)a.kb_total * rank / a.splits);
    const int kb1 = (int)((long long)a.kb_total * (rank + 1) / a.splits);
    const int nkb = kb1 - kb0;
    const int S = a.stages;
    const int ptiles = TN / kPanelN;                            // 128-channel panel tiles per CTA
    const uint32_t b_off = (uint32_t)(TMB * P) * kActTileBytes;  // expanded weights after the activation tiles
    const uint32_t pk_off = b_off + (uint32_t)TN * kBK;          // packed codes after the expanded weights
    const uint32_t pk_tile_bytes = WBITS * kPanelSubBytes;
    const uint32_t tx_bytes = (uint32_t)(TMB * P) * kActTileBytes + (uint32_t)ptiles * pk_tile_bytes;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bar_full[s]), 1);
            mbar_init(smem_u32(&bar_exp[s]), kEpiThreads / 32);
            mbar_init(smem_u32(&bar_empty[s]), 1);
        }
        mbar_init(smem_u32(&bar_acc), 1);
        fence_barrier_init();
        prefetch_tensormap(&qmap);
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(&tmem_slot), a.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    // Everything below may read what the previous kernel in the stream wrote.
    grid_dependency_wait();

    bool ok = true;
    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const size_t tile_stride = (size_t)a.kb_total * pk_tile_bytes;
            const uint8_t *wsrc = a.panels + (size_t)(n0 / kPanelN) * tile_stride;
            int issued = 0;
            for (int i = 0; i < nkb; ++i) {
                const int s = i % S;
                if (i >= S && !mbar_wait(smem_u32(&bar_empty[s]), ((i / S) - 1) & 1, kWaitBudget)) {
                    ok = false;
                    break;
                }
                const uint32_t st = base + (uint32_t)s * a.stage_bytes;
                const uint32_t full = smem_u32(&bar_full[s]);
                const int kb = kb0 + i;
                mbar_arrive_expect_tx(full, tx_bytes);
                for (int pt = 0; pt < ptiles; ++pt)
                    bulk_load(st + pk_off + pt * pk_tile_bytes, wsrc + pt * tile_stride + (size_t)kb * pk_tile_bytes,
                              pk_tile_bytes, full);
                for (int tb = 0; tb < TMB; ++tb)
                    for (int p = 0; p < P; ++p)
                        tma_load_3d(st + (tb * P + p) * kActTileBytes, &qmap, full, kb * kBK, t0 + tb * kBM, p);
                issued = i + 1;
            }
            if (!ok) {
                report(a.err, 1u);
                for (int i = (issued > S ? issued - S : 0); i < issued; ++i)   // let issued copies land first
                    mbar_wait(smem_u32(&bar_full[i % S]), (i / S) & 1, kWaitBudget);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(kBM, (uint32_t)TN);
            for (int i = 0; i < nkb; ++i) {
                const int s = i % S;
                const uint32_t ph = (i / S) & 1;
                if (!mbar_wait(smem_u32(&bar_full[s]), ph, kWaitBudget) || !mbar_wait(smem_u32(&bar_exp[s]), ph, kWaitBudget)) {
                    ok = false;
                    report(a.err, 1u);
                    break;
                }
                tc_fence_after();
                const uint32_t st = base + (uint32_t)s * a.stage_bytes;
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t bd = sw128_kmajor_desc(st + b_off + kk * 32);
                    for (int blk = 0; blk < TMB * P; ++blk) {
                        const uint64_t ad = sw128_kmajor_desc(st + blk * kActTileBytes + kk * 32);
                        mma_i8(tmem + (uint32_t)(blk * TN), ad, bd, idesc, (i | kk) != 0 ? 1u : 0u);
                    }
                }
                mma_commit(smem_u32(&bar_empty[s]));
            }
            mma_commit(smem_u32(&bar_acc));
        }
    } else {
        // ---------------- expanders ----------------
        const int e = threadIdx.x - 64;   // 0 .. 255
        for (int i = e; i < P * TMB * kBM; i += kEpiThreads) {
            const int p = i / (TMB * kBM), t = t0 + (i - p * TMB * kBM);
            s_qs[i] = t < a.M ? a.qs[p * a.qs_stride + t] : 0.f;
        }
        for (int i = e; i < TN; i += kEpiThreads) {
            const int n = n0 + i;
            s_alpha[i] = n < a.N ? a.alpha[n] : 0.f;
            s_bias[i] = (a.bias && n < a.N) ? a.bias[n] : 0.f;
        }
        for (int i = 0; i < nkb; ++i) {
            const int s = i % S;
            bool landed = mbar_wait(smem_u32(&bar_full[s]), (i / S) & 1, kWaitBudget);
            if (!__all_sync(0xFFFFFFFFu, landed)) {
                ok = false;
                if (lane == 0) report(a.err, 1u);
                break;
            }
            const uint32_t st = base + (uint32_t)s * a.stage_bytes;
            if (TN == 128) {      // two threads per channel row, four chunks each
                const int row = e & 127, half = e >> 7;
                expand_chunks<WBITS, 4>(st + pk_off, st + b_off, row, half * 4);
            } else {              // one thread per channel row of the two panel tiles
                // packed row of channel e: tile e / 128, row e % 128 (expand_chunks adds e * 16)
                const uint32_t pk = st + pk_off + (uint32_t)(e >> 7) * (pk_tile_bytes - kPanelSubBytes);
                expand_chunks<WBITS, 8>(pk, st + b_off, e, 0);
            }
            fence_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bar_exp[s]));
        }
    }

    // ---------------- epilogue (warps 2-9) ----------------
    const int quad = warp & 3;                  // the TMEM lane quarter this warp may access
    const int half = (warp - 2) >> 2;           // which of the two warps on this quarter
    const int row = quad * 32 + lane;           // token row within a 128-token block
    const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
    uint32_t red = base;                        // split-K exchange buffer (reuses the stage area)
    if (warp >= 2) {
        named_barrier_sync(1, kEpiThreads);     // s_qs / s_alpha / s_bias complete
        bool done = ok && mbar_wait(smem_u32(&bar_acc), 0, kWaitBudget);
        done = __all_sync(0xFFFFFFFFu, done);
        if (!done && ok && lane == 0) report(a.err, 1u);
        tc_fence_after();
        if (a.splits == 1) {
            if (done) {
                for (int tb = 0; tb < TMB; ++tb) {
                    const int t = t0 + tb * kBM + row;
                    float s[P];
#pragma unroll
                    for (int p = 0; p < P; ++p) s[p] = s_qs[p * TMB * kBM + tb * kBM + row];
                    // 16-column chunks of this block, alternating between the two warps of the quarter
                    for (int c = half * 16; c < TN; c += 32) {
                        uint32_t v[P][16];
#pragma unroll
                        for (int p = 0; p < P; ++p) tmem_ld16(lane_addr + (uint32_t)((tb * P + p) * TN + c), v[p]);
                        tmem_wait_ld();
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
            // partials -> red: [block = tb * P + p][channel group g = c / 4][row][4] int32 (16-byte rows)
            const int blocks = TMB * P;
            for (int blk = 0; blk < blocks; ++blk) {
                for (int c = half * 16; c < TN; c += 32) {
                    uint32_t v[16];
                    if (done) {
                        tmem_ld16(lane_addr + (uint32_t)(blk * TN + c), v);
                        tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) v[j] = 0;
                    }
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        const uint32_t addr = red + (uint32_t)((((blk * (TN / 4) + c / 4 + g) * kBM) + row) * 16);
                        st_shared_v4(addr, v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
                    }
                }
            }
        }
    }

    if (a.splits > 1) {
        cluster_sync_all();  // every CTA's partials are in its shared memory
        if (warp >= 2) {
            // this rank finishes channel groups [g_lo, g_hi) of the tile; the quarter's two warps alternate groups
            const int groups = TN / 4;
            const int per = (groups + a.splits - 1) / a.splits;
            const int g_lo = rank * per, g_hi = min(groups, g_lo + per);
            for (int tb = 0; tb < TMB; ++tb) {
                const int t = t0 + tb * kBM + row;
                float s[P];
#pragma unroll
                for (int p = 0; p < P; ++p) s[p] = s_qs[p * TMB * kBM + tb * kBM + row];
                if (t >= a.M) continue;
                for (int g = g_lo + half; g < g_hi; g += 2) {
                    int accv[P][4];
#pragma unroll
                    for (int p = 0; p < P; ++p) {
                        const uint32_t off = red + (uint32_t)(((((tb * P + p) * groups + g) * kBM) + row) * 16);
                        int4 sum = make_int4(0, 0, 0, 0);
                        for (int r0 = 0; r0 < a.splits; r0 += 4) {   // four peers' loads in flight at a time
                            int4 part[4];
#pragma unroll
                            for (int r = 0; r < 4; ++r)
                                if (r0 + r < a.splits) part[r] = ld_cluster_v4(map_to_rank(off, (uint32_t)(r0 + r)));
#pragma unroll
                            for (int r = 0; r < 4; ++r)
                                if (r0 + r < a.splits) {
                                    sum.x += part[r].x;
                                    sum.y += part[r].y;
                                    sum.z += part[r].z;
                                    sum.w += part[r].w;
                                }
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
        cluster_sync_all();  // no CTA leaves while a peer still reads its shared memory
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
