// gemm_reg_kernel.cuh - the low-bit GEMM for small M with register operands: warp-level tensor-core MMAs
// (mma.sync m16n8k32, INT8 x INT8 -> INT32) whose weight operand is expanded from the packed panels in registers.
//
// With a few dozen to a hundred tokens a launch is latency-bound, and the tcgen05 kernels' fixed costs dominate it:
// tensor-memory allocation, mbarrier set-up, a TMA round trip for a whole 128-row activation block per CTA, the
// weight tile expanded into shared memory behind an async-proxy fence, and a chain of issue-paced MMAs from one
// thread. Here nothing is staged: every warp loads its operands straight from global memory into registers, a few
// double steps ahead, and issues its own MMAs.
//
// Operands. The weights are the MMA's A operand (16 channels x 32 k), the tokens its B operand (32 k x 8 rows). An
// integer dot product does not depend on the order of its K terms as long as both operands use the same order, so
// k is walked in double steps of 64 (two MMAs) ordered to suit the panels and 16-byte loads: lane (g, t) (g = lane /
// 4, t = lane % 4) holds codes 16t .. 16t+15 of its channel's double step and bytes 16t .. 16t+15 of its token row
// (one 16-byte load); MMA h (0, 1) of the double step takes codes / bytes 16t + 8h .. 16t + 8h + 7, the first four in
// its first A register of that row and first B register, the next four in the second. With the PTX fragment layout
// (A: registers 0 / 2 = row g at logical columns 4t .. 4t+3 / 16+4t .. 16+4t+3, registers 1 / 3 = row g + 8;
// B: registers 0 / 1 = logical rows 4t .. 4t+3 / 16+4t .. 16+4t+3 of column g) logical column 4t + i of MMA h is
// k = 16t + 8h + i of the double step and 16 + 4t + i is 16t + 8h + 4 + i, for both operands. In the panels, 1-bit
// word w of a channel row holds codes 32w .. 32w+31 with code c at bit 4 (c % 8) + c / 8 (c within the word), so
// this lane's codes of double step s lie in word 2s + t/2 and those of MMA h are the nibbles of
// (word >> (2 (t % 2) + h)) & 0x11111111; a 2-bit word holds 16 codes with field f at bits 4 (f % 8) + 2 (f / 8), so
// the lane's codes are word 4s + t and those of MMA h the nibbles of (word >> 2h) & 0x33333333. Either way two
// byte-permute lookups per register pair expand them (the tcgen05 expanders' tables).
//
// Work split. A CTA owns CN consecutive channels x TT tokens (all parts of those tokens: rows r = p * TT + token,
// R = 8 * RG rows). Its 8 warps are KS K-slices x (8 / KS) channel groups: a warp computes 16 * CG channels x all R
// rows over its slice of the double steps, 2 x CG x RG MMAs per double step with INT32 accumulators in registers.
// Its loads run D double steps ahead of its MMAs (a ring of D register sets; a slot is refilled right after its double
// step is used). The weights do not depend on the previous kernel of the stream, so the ring's first weight loads are
// issued before griddepcontrol.wait (programmatic dependent launch overlaps them with that kernel's tail); the
// activations, which that kernel may still be writing, are read with ordinary loads after the wait. The K-slices'
// partial sums meet in shared memory ([slice][row][channel], rows padded by 4 words so the fragment stores do not
// collide) and every thread sums them in slice order (exact INT32: the order cannot change the result) and finishes
// (token, channel) outputs with the tensor-core kernels' finish_value, so the outputs equal theirs bit for bit.
#pragma once

#include "gemm_kernel.cuh"

namespace kea {

constexpr int kRegThreads = 256;
constexpr int kRegWarps = kRegThreads / 32;
constexpr int kRegPad = 4;   // words of padding per shared-memory row of partial sums

// Dynamic shared memory of a launch: the K-slices' partial sums.
__host__ __device__ inline int reg_smem_bytes(int ks, int rows, int cn) { return ks * rows * (cn + kRegPad) * 4; }

struct RegArgs {
    const int8_t *q;
    long long q_stride;      // elements between parts
    int ldq;
    const float *qs;
    long long qs_stride;
    const uint8_t *panels;
    const float *alpha;
    const float *bias;
    void *y;
    long long ldy;
    int y_f16;
    int *acc;
    long long ld_acc, acc_stride;
    const float *res;        // residual FP32 [M][ld_res] or null: y = res + res_scale * value
    long long ld_res;
    float res_scale;
    int M, N, K, kb_total;
    int ks;                  // K-slices among the 8 warps: 1, 2, 4 or 8
    int tt;                  // tokens per CTA (rows / parts)
    int flags;
};

KEA_DEVI void mma_s8_m16n8k32(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Bytes 0 .. v - 1 of a word kept (v <= 0: none, v >= 4: all).
KEA_DEVI uint32_t keep_bytes(uint32_t w, int v) {
    return v >= 4 ? w : (v <= 0 ? 0u : w & ((1u << (8 * v)) - 1u));
}

template <int WBITS, int P, int CG, int RG, int D>
__global__ void __launch_bounds__(kRegThreads, 2) lowbit_gemm_reg_kernel(const RegArgs a) {
    extern __shared__ __align__(16) int rsm[];
    grid_launch_dependents();
    constexpr int R = 8 * RG;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    const int KS = a.ks, CW = kRegWarps / KS;
    const int kw = warp % KS, cw = warp / KS;
    const int CN = 16 * CG * CW;
    const int c0 = blockIdx.x * CN;
    const int m0 = blockIdx.y * a.tt;

    // this warp's double k-steps (64 k each, two MMAs)
    const int steps = (a.K + 63) / 64;
    const int per = (steps + KS - 1) / KS;
    const int s0 = min(steps, kw * per), s1 = min(steps, s0 + per);

    // weight words: channel rows c0 + 16 (cw CG + cg) + g (+ 8); this lane's word of double step s is
    // 2s + t / 2 (1-bit) or 4s + t (2-bit)
    const uint32_t *pw = reinterpret_cast<const uint32_t *>(a.panels);
    const size_t tile_words = (size_t)a.kb_total * 4 * WBITS * 128;
    const uint32_t *wrow[CG][2];
#pragma unroll
    for (int cg = 0; cg < CG; ++cg)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int n = c0 + 16 * (cw * CG + cg) + g + 8 * h;   // < ceil(N / 128) * 128: inside the panels
            wrow[cg][h] = pw + (size_t)(n >> 7) * tile_words + (n & 127) + (WBITS == 1 ? (t >> 1) : t) * 128;
        }
    constexpr int WPS = 2 * WBITS;   // panel words per double step and channel row
    const int wshift = WBITS == 1 ? 2 * (t & 1) : 0;
    const uint32_t table = WBITS == 1 ? kSignTable : kTernaryTable;

    // activation rows: row 8 rg + g of the CTA (part r / tt, token m0 + r % tt), bytes 16t .. 16t+15 of each
    // double step
    const int8_t *qrow[RG];
#pragma unroll
    for (int rg = 0; rg < RG; ++rg) {
        const int r = 8 * rg + g, p = r / a.tt, m = m0 + r % a.tt;
        qrow[rg] = (p < P && m < a.M) ? a.q + p * a.q_stride + (long long)m * a.ldq + 16 * t : nullptr;
    }

    uint32_t wr[D][CG][2];
    uint4 br[D][RG];
#pragma unroll
    for (int d = 0; d < D; ++d) {
        const int s = s0 + d;
#pragma unroll
        for (int cg = 0; cg < CG; ++cg)
#pragma unroll
            for (int h = 0; h < 2; ++h) wr[d][cg][h] = s < s1 ? __ldg(wrow[cg][h] + (size_t)s * WPS * 128) : 0u;
    }
    grid_dependency_wait();
#pragma unroll
    for (int d = 0; d < D; ++d) {
        const int s = s0 + d;
        const bool live = s < s1 && 64 * s + 16 * t < a.K;
#pragma unroll
        for (int rg = 0; rg < RG; ++rg)
            br[d][rg] = (live && qrow[rg]) ? *reinterpret_cast<const uint4 *>(qrow[rg] + 64 * s)
                                           : make_uint4(0u, 0u, 0u, 0u);
    }

    int acc[CG][RG][4];
#pragma unroll
    for (int cg = 0; cg < CG; ++cg)
#pragma unroll
        for (int rg = 0; rg < RG; ++rg)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[cg][rg][i] = 0;

    for (int base = s0; base < s1; base += D) {
#pragma unroll
        for (int d = 0; d < D; ++d) {
            const int s = base + d;
            if (s >= s1) break;
            const int valid = a.K - (64 * s + 16 * t);   // codes at k >= K weigh 0 (a 1-bit zero code reads -1)
#pragma unroll
            for (int half = 0; half < 2; ++half) {   // codes 16t + 8 half .. + 7: the double step's MMA `half`
                uint32_t af[CG][4];
#pragma unroll
                for (int cg = 0; cg < CG; ++cg) {
                    uint32_t sel0, sel1;
                    if constexpr (WBITS == 1) {
                        sel0 = (wr[d][cg][0] >> (wshift + half)) & 0x11111111u;
                        sel1 = (wr[d][cg][1] >> (wshift + half)) & 0x11111111u;
                    } else {
                        sel0 = (wr[d][cg][0] >> (2 * half)) & 0x33333333u;
                        sel1 = (wr[d][cg][1] >> (2 * half)) & 0x33333333u;
                    }
                    af[cg][0] = lookup4(table, sel0);
                    af[cg][2] = lookup4(table, sel0 >> 16);
                    af[cg][1] = lookup4(table, sel1);
                    af[cg][3] = lookup4(table, sel1 >> 16);
                }
                const int v = valid - 8 * half;
                if (v < 8) {
#pragma unroll
                    for (int cg = 0; cg < CG; ++cg) {
                        af[cg][0] = keep_bytes(af[cg][0], v);
                        af[cg][1] = keep_bytes(af[cg][1], v);
                        af[cg][2] = keep_bytes(af[cg][2], v - 4);
                        af[cg][3] = keep_bytes(af[cg][3], v - 4);
                    }
                }
#pragma unroll
                for (int cg = 0; cg < CG; ++cg)
#pragma unroll
                    for (int rg = 0; rg < RG; ++rg)
                        mma_s8_m16n8k32(acc[cg][rg], af[cg], half ? br[d][rg].z : br[d][rg].x,
                                        half ? br[d][rg].w : br[d][rg].y);
            }
            // refill this slot with double step s + D
            const int sn = s + D;
#pragma unroll
            for (int cg = 0; cg < CG; ++cg)
#pragma unroll
                for (int h = 0; h < 2; ++h) wr[d][cg][h] = sn < s1 ? __ldg(wrow[cg][h] + (size_t)sn * WPS * 128) : 0u;
            const bool live = sn < s1 && 64 * sn + 16 * t < a.K;
#pragma unroll
            for (int rg = 0; rg < RG; ++rg)
                br[d][rg] = (live && qrow[rg]) ? *reinterpret_cast<const uint4 *>(qrow[rg] + 64 * sn)
                                               : make_uint4(0u, 0u, 0u, 0u);
        }
    }

    // partial sums of this K-slice: D fragment (channel g / g + 8, rows 2t / 2t + 1 of the tile)
    const int ld = CN + kRegPad;
    int *part = rsm + kw * R * ld;
#pragma unroll
    for (int cg = 0; cg < CG; ++cg)
#pragma unroll
        for (int rg = 0; rg < RG; ++rg) {
            const int ch = 16 * (cw * CG + cg) + g, r = 8 * rg + 2 * t;
            part[r * ld + ch] = acc[cg][rg][0];
            part[(r + 1) * ld + ch] = acc[cg][rg][1];
            part[r * ld + ch + 8] = acc[cg][rg][2];
            part[(r + 1) * ld + ch + 8] = acc[cg][rg][3];
        }
    __syncthreads();

    const bool has_bias = a.bias != nullptr;
    const bool small = a.K <= 32768;
    for (int i = threadIdx.x; i < a.tt * CN; i += kRegThreads) {
        const int tt = i / CN, ch = i - tt * CN;
        const int m = m0 + tt, n = c0 + ch;
        if (m >= a.M || n >= a.N) continue;
        int tot[3] = {0, 0, 0};
        float s[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < P; ++p) {
            int v = 0;
            for (int w = 0; w < KS; ++w) v += rsm[(w * R + p * a.tt + tt) * ld + ch];
            tot[p] = v;
            s[p] = a.qs[p * a.qs_stride + m];
        }
        float v = finish_value(tot[0], tot[1], tot[2], s[0], s[1], s[2], P, a.flags, __ldg(a.alpha + n), has_bias,
                               has_bias ? __ldg(a.bias + n) : 0.f, small);
        if (a.res) v = __fadd_rn(a.res[(long long)m * a.ld_res + n], __fmul_rn(a.res_scale, v));
        if (a.y_f16)
            reinterpret_cast<__half *>(a.y)[(long long)m * a.ldy + n] = __float2half_rn(v);
        else
            reinterpret_cast<float *>(a.y)[(long long)m * a.ldy + n] = v;
        if (a.acc) {
#pragma unroll
            for (int p = 0; p < P; ++p) a.acc[p * a.acc_stride + (long long)m * a.ld_acc + n] = tot[p];
        }
    }
}

}  // namespace kea
