// gemm_kernel.cuh - the low-bit GEMM for sm_100a.
//
// One CTA computes a 128-channel x `bt`-token output tile over the k128 blocks of its split:
//   warp 0     producer: one cp.async.bulk of the packed weight panel (wbits x 2 KB) and one TMA tile per
//              activation part (bt rows x 128 int8, 128-byte swizzle) per stage, both on the stage's
//              `full` mbarrier;
//   warp 1     allocates tensor memory; one thread issues tcgen05.mma.kind::i8 (M = 128 channels,
//              N = bt tokens, K = 32) with A = expanded weights and B = activations, INT32 accumulators in
//              TMEM (one bt-column block per part), and frees each stage with tcgen05.commit;
//   warps 2-5  expand the packed codes of one channel row each (1 bit -> int8 +-1, 2 bits -> int8
//              -1/0/+1) into the 128-byte-swizzled K-major A tile, then run the epilogue.
// Split-K: the `splits` CTAs of a thread-block cluster share one output tile; each copies its INT32
// partials TMEM -> its own shared memory, and after a cluster barrier every CTA sums a slice of tokens
// across the cluster through distributed shared memory (exact INT32, order-free) and finishes it.
// Epilogue: comb_P, alpha / bias, optional SiLU, FP32 or FP16 stores, optional INT32 accumulator stores.
#pragma once

#include <cuda_fp16.h>

#include "ptx.cuh"

namespace kea {

constexpr int kThreads = 192;
constexpr int kTileN = 128;          // output channels per CTA (tcgen05 M)
constexpr int kBK = 128;             // k per stage: one 128-byte swizzled row of int8
constexpr int kMaxStages = 8;
constexpr int kExpBytes = kTileN * kBK;   // expanded weight tile per stage (16 KB)
constexpr int kPanelRowBytes = 16;        // one row of one panel sub-block
constexpr int kPanelSubBytes = kTileN * kPanelRowBytes;  // 2 KB per sub-block (wbits sub-blocks per k128)
constexpr long long kWaitBudget = 4000000000LL;          // SM clocks (about 2 s) before a wait gives up

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
    int parts, bt, splits, stages, kb_total;
    int flags;
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

// Expands channel row `row` of one k128 stage: packed codes at `pk` (wbits sub-blocks of [128 rows][16 B])
// into the int8 A tile at `dst` (row r at r * 128, 16-byte chunk c stored at chunk c ^ (r & 7)).
template <int WBITS>
KEA_DEVI void expand_row(uint32_t pk, uint32_t dst, int row) {
    uint32_t w[4 * WBITS];
    {
        const uint4 v = ld_shared_v4(pk + row * kPanelRowBytes);
        w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    }
    if constexpr (WBITS == 2) {
        const uint4 v = ld_shared_v4(pk + kPanelSubBytes + row * kPanelRowBytes);
        w[4] = v.x; w[5] = v.y; w[6] = v.z; w[7] = v.w;
    }
    const uint32_t rowbase = dst + row * 128;
    const uint32_t sw = row & 7;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint32_t o0, o1, o2, o3;
        if constexpr (WBITS == 1) {
            // codes 16c .. 16c+15 are packed bytes 2c and 2c+1 (LSB first)
            const uint32_t word = w[c >> 1];
            const uint32_t r0 = byte_in_all_lanes(word, 2 * (c & 1)), r1 = byte_in_all_lanes(word, 2 * (c & 1) + 1);
            o0 = sign_lanes(lane_bits(r0, 0x08040201u));
            o1 = sign_lanes(lane_bits(r0, 0x80402010u));
            o2 = sign_lanes(lane_bits(r1, 0x08040201u));
            o3 = sign_lanes(lane_bits(r1, 0x80402010u));
        } else {
            // codes 16c .. 16c+15: sub-block c / 4 (64 codes each), packed word c % 4 of it (4 codes per byte)
            const uint32_t word = w[(c >> 2) * 4 + (c & 3)];
            o0 = ternary_lanes(byte_in_all_lanes(word, 0));
            o1 = ternary_lanes(byte_in_all_lanes(word, 1));
            o2 = ternary_lanes(byte_in_all_lanes(word, 2));
            o3 = ternary_lanes(byte_in_all_lanes(word, 3));
        }
        st_shared_v4(rowbase + ((c ^ sw) << 4), o0, o1, o2, o3);
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

KEA_DEVI void store_output(const GemmArgs &a, int t, int n, float v, int a0, int a1, int a2) {
    const long long off = (long long)t * a.ldy + n;
    if (a.y_f16)
        reinterpret_cast<__half *>(a.y)[off] = __float2half_rn(v);
    else
        reinterpret_cast<float *>(a.y)[off] = v;
    if (a.acc) {
        const long long o = (long long)t * a.ld_acc + n;
        a.acc[o] = a0;
        if (a.parts > 1) a.acc[a.acc_stride + o] = a1;
        if (a.parts > 2) a.acc[2 * a.acc_stride + o] = a2;
    }
}

KEA_DEVI void named_barrier_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

KEA_DEVI void report(uint32_t *err, uint32_t bits) { atomicOr(err ? err : &g_device_error, bits); }

template <int WBITS>
__global__ void __launch_bounds__(kThreads, 1) lowbit_gemm_kernel(const __grid_constant__ CUtensorMap qmap, const GemmArgs a) {
    extern __shared__ uint8_t dyn_smem[];
    __shared__ __align__(8) uint64_t bar_full[kMaxStages];
    __shared__ __align__(8) uint64_t bar_exp[kMaxStages];
    __shared__ __align__(8) uint64_t bar_empty[kMaxStages];
    __shared__ __align__(8) uint64_t bar_acc;
    __shared__ uint32_t tmem_slot;
    __shared__ float s_qs[3 * 256];

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t raw = smem_u32(dyn_smem);
    const uint32_t base = (raw + 1023u) & ~1023u;   // 128-byte swizzle atoms need 1024-byte alignment
    const int tile_n = blockIdx.x;
    const int n0 = tile_n * kTileN, t0 = blockIdx.y * a.bt;
    const int rank = a.splits > 1 ? (int)cluster_ctarank() : 0;
    const int kb0 = (int)((long long)a.kb_total * rank / a.splits);
    const int kb1 = (int)((long long)a.kb_total * (rank + 1) / a.splits);
    const int nkb = kb1 - kb0;
    const int S = a.stages;
    const uint32_t act_off = kExpBytes;
    const uint32_t act_part_bytes = (uint32_t)a.bt * 128u;
    const uint32_t pk_off = kExpBytes + (uint32_t)a.parts * act_part_bytes;
    const uint32_t tx_bytes = (uint32_t)a.parts * act_part_bytes + WBITS * kPanelSubBytes;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(smem_u32(&bar_full[s]), 1);
            mbar_init(smem_u32(&bar_exp[s]), 4);
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
            const uint8_t *wsrc = a.panels + (size_t)tile_n * a.kb_total * (WBITS * kPanelSubBytes);
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
                bulk_load(st + pk_off, wsrc + (size_t)kb * (WBITS * kPanelSubBytes), WBITS * kPanelSubBytes, full);
                for (int p = 0; p < a.parts; ++p) tma_load_3d(st + act_off + p * act_part_bytes, &qmap, full, kb * kBK, t0, p);
                issued = i + 1;
            }
            if (!ok) {
                report(a.err, 1u);
                // let the copies already issued land before this CTA may exit
                for (int i = (issued > S ? issued - S : 0); i < issued; ++i)
                    mbar_wait(smem_u32(&bar_full[i % S]), (i / S) & 1, kWaitBudget);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(kTileN, (uint32_t)a.bt);
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
                for (int p = 0; p < a.parts; ++p) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = sw128_kmajor_desc(st + kk * 32);
                        const uint64_t bd = sw128_kmajor_desc(st + act_off + p * act_part_bytes + kk * 32);
                        mma_i8(tmem + (uint32_t)(p * a.bt), ad, bd, idesc, (i | kk) != 0 ? 1u : 0u);
                    }
                }
                mma_commit(smem_u32(&bar_empty[s]));
            }
            mma_commit(smem_u32(&bar_acc));
        }
    } else {
        // ---------------- expanders ----------------
        const int e = threadIdx.x - 64;  // channel row of the tile
        for (int i = e; i < a.parts * a.bt; i += 128) {
            const int p = i / a.bt, t = t0 + (i - p * a.bt);
            s_qs[i] = t < a.M ? a.qs[p * a.qs_stride + t] : 0.f;
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
            expand_row<WBITS>(st + pk_off, st, e);
            fence_async_shared();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&bar_exp[s]));
        }
    }

    // ---------------- epilogue (warps 2-5) ----------------
    const int quad = warp & 3;            // the TMEM lane quarter this warp may access
    const int row = quad * 32 + lane;     // channel within the tile
    const int n = n0 + row;
    const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
    const bool has_bias = a.bias != nullptr;
    int *red = reinterpret_cast<int *>(dyn_smem + (base - raw));
    if (warp >= 2) {
        named_barrier_sync(1, 128);  // s_qs complete
        bool done = ok && mbar_wait(smem_u32(&bar_acc), 0, kWaitBudget);
        done = __all_sync(0xFFFFFFFFu, done);
        if (!done && ok && lane == 0) report(a.err, 1u);
        tc_fence_after();
        if (a.splits == 1) {
            const float alpha = n < a.N ? a.alpha[n] : 0.f;
            const float bias = (has_bias && n < a.N) ? a.bias[n] : 0.f;
            for (int j0 = 0; done && j0 < a.bt && t0 + j0 < a.M; j0 += 16) {
                uint32_t v0[16], v1[16], v2[16];
                tmem_ld16(lane_addr + j0, v0);
                if (a.parts > 1) tmem_ld16(lane_addr + a.bt + j0, v1);
                if (a.parts > 2) tmem_ld16(lane_addr + 2 * a.bt + j0, v2);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = t0 + j0 + j;
                    if (t < a.M && n < a.N) {
                        const int a0 = (int)v0[j], a1 = a.parts > 1 ? (int)v1[j] : 0, a2 = a.parts > 2 ? (int)v2[j] : 0;
                        const int c = j0 + j;
                        const float val = finish_value(a0, a1, a2, s_qs[c], a.parts > 1 ? s_qs[a.bt + c] : 0.f,
                                                       a.parts > 2 ? s_qs[2 * a.bt + c] : 0.f, a.parts, a.flags, alpha,
                                                       has_bias, bias);
                        store_output(a, t, n, val, a0, a1, a2);
                    }
                }
            }
        } else {
            // partial accumulators -> red[column][row] in this CTA's shared memory
            const int cols = a.parts * a.bt;
            for (int c0 = 0; c0 < cols; c0 += 16) {
                uint32_t v[16];
                if (done) {
                    tmem_ld16(lane_addr + c0, v);
                    tmem_wait_ld();
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = 0;
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) red[(c0 + j) * kTileN + row] = (int)v[j];
            }
        }
    }

    if (a.splits > 1) {
        cluster_sync_all();  // every CTA's partials are in its shared memory
        if (warp >= 2) {
            const float alpha = n < a.N ? a.alpha[n] : 0.f;
            const float bias = (has_bias && n < a.N) ? a.bias[n] : 0.f;
            uint32_t peer[16];
            const uint32_t red_addr = smem_u32(red);
#pragma unroll
            for (int r = 0; r < 16; ++r) peer[r] = r < a.splits ? map_to_rank(red_addr, (uint32_t)r) : 0u;
            const int per = (a.bt + a.splits - 1) / a.splits;
            const int j_lo = rank * per, j_hi = min(a.bt, j_lo + per);
            for (int j = j_lo; j < j_hi; ++j) {
                const int t = t0 + j;
                if (t >= a.M) break;
                int sum[3] = {0, 0, 0};
#pragma unroll
                for (int p = 0; p < 3; ++p) {
                    if (p < a.parts) {
                        const uint32_t off = (uint32_t)(((p * a.bt + j) * kTileN + row) * 4);
#pragma unroll
                        for (int r = 0; r < 16; ++r)
                            if (r < a.splits) sum[p] += ld_cluster_s32(peer[r] + off);
                    }
                }
                if (n < a.N) {
                    const float val = finish_value(sum[0], sum[1], sum[2], s_qs[j], a.parts > 1 ? s_qs[a.bt + j] : 0.f,
                                                   a.parts > 2 ? s_qs[2 * a.bt + j] : 0.f, a.parts, a.flags, alpha,
                                                   has_bias, bias);
                    store_output(a, t, n, val, sum[0], sum[1], sum[2]);
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
