// gemv_kernel.cuh - the low-bit GEMM for a handful of tokens (decode-sized M), on the CUDA cores.
//
// With a few tokens the tensor-core kernels are latency-bound on their own set-up (tensor memory, mbarriers, a TMA
// round trip, a chain of serial MMA instructions of which at most 16 of 128 rows carry data). Here each CTA owns CH
// consecutive output channels (a lane's channel is lane % CH) and its 8 warps, times 32 / CH lane groups, split the
// channel's code words into contiguous slices. Every lane loads its slice of packed code words straight from the
// panels (the CH lanes of a group read consecutive words: coalesced) BEFORE waiting on the previous kernel of the
// stream - the weights do not depend on it - so with programmatic dependent launch the weight fetch overlaps that
// kernel's tail. Each lane then expands its code words in registers with the tensor-core expanders' byte-permute
// tables and accumulates INT8 x {-1, 0, +1} products for every token and part with dp4a (exact INT32), reading
// activations 16 bytes at a time straight from global memory (the lanes of a group read the same bytes: one
// broadcast), four rows' loads issued before their products. The slices are summed in shared memory in a fixed
// order, and the FP32 epilogue is the tensor-core kernels' finish_value (one IEEE rounding per operation), so results
// are bit-identical to them. (Staging the CTA's activation rows in shared memory first was measured slower: the
// CTA-wide barrier after the copy serialises what the direct loads overlap.)
#pragma once

#include "gemm_kernel.cuh"

namespace kea {

constexpr int kGemvThreads = 256;
constexpr int kGemvMaxM = 16;
constexpr int kGemvWords = 8;    // code words a lane holds in registers per round (two rounds in flight)
constexpr int kGemvRowBatch = 4; // activation rows whose loads are issued together
constexpr int kGemvMaxSmem = 48 * 1024;
constexpr int kGemvCtasPerSm = 3;  // register budget: three CTAs resident per SM

// Dynamic shared memory of a launch: the slice sums, [warp][row][channel] INT32.
__host__ __device__ inline int gemv_smem_bytes(int rows, int ch) { return (kGemvThreads / 32) * rows * ch * 4; }

struct GemvArgs {
    const int8_t *q;
    long long q_stride;          // elements between parts
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
    int M, N, K, kb_total;
    int ch;                      // channels per CTA: 32, 16 or 8
    int flags;
    const float *res;            // residual FP32 [M][ld_res] or null: y = res + res_scale * value
    long long ld_res;
    float res_scale;
    uint32_t *err;
};


template <int WBITS, int P, int MT>
__global__ void __launch_bounds__(kGemvThreads, kGemvCtasPerSm) lowbit_gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(16) uint8_t gsm[];
    // the next kernel of the stream may start its own weight prefetch now; its reads of our output wait for us
    grid_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int CH = a.ch, groups = 32 / CH;
    const int c = lane % CH, grp = lane / CH;
    const int n = blockIdx.x * CH + c;
    // Panel word w of a channel row (k-block w / (4 WBITS), sub-block and word within it) holds codes w * CPW ..
    // + CPW - 1 of the row, so the words that carry codes below K are 0 .. ceil(K / CPW) - 1.
    constexpr int CPW = 32 / WBITS;
    const int words = (a.K + CPW - 1) / CPW;
    const int slices = (kGemvThreads / 32) * groups;
    const int per = (words + slices - 1) / slices;
    const int w0 = min(words, (warp * groups + grp) * per), w1 = min(words, w0 + per);
    const bool live = n < a.N;
    const uint32_t *tw = reinterpret_cast<const uint32_t *>(a.panels) + (size_t)(n >> 7) * a.kb_total * 4 * WBITS * 128 +
                         (n & 127);

    uint32_t cur[kGemvWords], nxt[kGemvWords];
#pragma unroll
    for (int j = 0; j < kGemvWords; ++j) cur[j] = (live && w0 + j < w1) ? __ldg(tw + (size_t)(w0 + j) * 128) : 0u;
    grid_dependency_wait();

    const int rows = P * a.M;
    int acc[P][MT];
#pragma unroll
    for (int p = 0; p < P; ++p)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[p][m] = 0;

    for (int wb = w0; wb < w1; wb += kGemvWords) {
        const bool more = wb + kGemvWords < w1;   // the next round's words, loaded while this round computes
#pragma unroll
        for (int j = 0; j < kGemvWords; ++j) {
            const int w = wb + kGemvWords + j;
            nxt[j] = (more && live && w < w1) ? __ldg(tw + (size_t)w * 128) : 0u;
        }
#pragma unroll
        for (int j = 0; j < kGemvWords; ++j) {
            const int w = wb + j;
            if (w >= w1) break;
            const uint32_t code = cur[j];
            const int k0 = w * CPW;
            uint32_t e[CPW / 4];   // expanded int8 weights, four per register: codes k0 + 4 i .. k0 + 4 i + 3
            if constexpr (WBITS == 1) {
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint32_t sel = (code >> t) & 0x11111111u;   // codes 8 t .. 8 t + 7, one per nibble
                    e[2 * t] = lookup4(kSignTable, sel);
                    e[2 * t + 1] = lookup4(kSignTable, sel >> 16);
                }
            } else {
                const uint32_t lo = code & 0x33333333u, hi = (code >> 2) & 0x33333333u;
                e[0] = lookup4(kTernaryTable, lo);
                e[1] = lookup4(kTernaryTable, lo >> 16);
                e[2] = lookup4(kTernaryTable, hi);
                e[3] = lookup4(kTernaryTable, hi >> 16);
            }
            const int valid = a.K - k0;   // >= 1; codes at k >= K weigh 0 (a 1-bit zero code would read -1)
            if (valid < CPW) {
#pragma unroll
                for (int i = 0; i < CPW / 4; ++i) {
                    const int lim = valid - 4 * i;
                    e[i] = lim <= 0 ? 0u : (lim >= 4 ? e[i] : e[i] & ((1u << (8 * lim)) - 1u));
                }
            }
            // 16-byte activation chunks: a chunk that starts below K lies inside the row (ldq is a multiple of 16
            // and >= K) and its bytes at k >= K meet zero weights; chunks starting at or past K are not read
#pragma unroll
            for (int r0 = 0; r0 < P * MT; r0 += kGemvRowBatch) {
                uint4 v[kGemvRowBatch][CPW / 16];
#pragma unroll
                for (int b = 0; b < kGemvRowBatch; ++b) {
                    const int p = (r0 + b) / MT, m = (r0 + b) % MT;
                    const bool row_live = (r0 + b < P * MT) && m < a.M;
                    const uint4 *row = reinterpret_cast<const uint4 *>(a.q + p * a.q_stride + (long long)m * a.ldq + k0);
#pragma unroll
                    for (int h = 0; h < CPW / 16; ++h)
                        v[b][h] = (row_live && 16 * h < valid) ? row[h] : make_uint4(0, 0, 0, 0);
                }
#pragma unroll
                for (int b = 0; b < kGemvRowBatch; ++b) {
                    if (r0 + b < P * MT && (r0 + b) % MT < a.M) {
                        const int p = (r0 + b) / MT, m = (r0 + b) % MT;
                        int s = acc[p][m];
#pragma unroll
                        for (int h = 0; h < CPW / 16; ++h) {
                            s = __dp4a((int)e[4 * h], (int)v[b][h].x, s);
                            s = __dp4a((int)e[4 * h + 1], (int)v[b][h].y, s);
                            s = __dp4a((int)e[4 * h + 2], (int)v[b][h].z, s);
                            s = __dp4a((int)e[4 * h + 3], (int)v[b][h].w, s);
                        }
                        acc[p][m] = s;
                    }
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kGemvWords; ++j) cur[j] = nxt[j];
    }
    // sum the lane groups of the warp (same channel, other slices), then the warps through shared memory
    int *red = reinterpret_cast<int *>(gsm);   // [warp][row][channel]
#pragma unroll
    for (int p = 0; p < P; ++p)
#pragma unroll
        for (int m = 0; m < MT; ++m) {
            if (m < a.M) {
                int v = acc[p][m];
                for (int o = CH; o < 32; o <<= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
                if (grp == 0) red[(warp * rows + p * a.M + m) * CH + c] = v;
            }
        }
    __syncthreads();
    for (int i = threadIdx.x; i < a.M * CH; i += kGemvThreads) {
        const int m = i / CH, cc = i - m * CH, nn = blockIdx.x * CH + cc;
        if (nn >= a.N) continue;
        int tot[3] = {0, 0, 0};
        float s[3] = {0.f, 0.f, 0.f};
#pragma unroll
        for (int p = 0; p < P; ++p) {
            int v = 0;
#pragma unroll
            for (int w = 0; w < kGemvThreads / 32; ++w) v += red[(w * rows + p * a.M + m) * CH + cc];
            tot[p] = v;
            s[p] = a.qs[p * a.qs_stride + m];
        }
        const bool has_bias = a.bias != nullptr;
        float v = finish_value(tot[0], tot[1], tot[2], s[0], s[1], s[2], P, a.flags, __ldg(a.alpha + nn), has_bias,
                               has_bias ? __ldg(a.bias + nn) : 0.f, a.K <= 32768);
        if (a.res) v = __fadd_rn(a.res[(long long)m * a.ld_res + nn], __fmul_rn(a.res_scale, v));
        if (a.y_f16)
            reinterpret_cast<__half *>(a.y)[(long long)m * a.ldy + nn] = __float2half_rn(v);
        else
            reinterpret_cast<float *>(a.y)[(long long)m * a.ldy + nn] = v;
        if (a.acc) {
#pragma unroll
            for (int p = 0; p < P; ++p) a.acc[p * a.acc_stride + (long long)m * a.ld_acc + nn] = tot[p];
        }
    }
}

}  // namespace kea
