// aux_kernels.cuh - the two kernels beside the GEMM: panel preparation (once per layer, at load) and the
// residual INT8 activation quantizer (once per projection call).
#pragma once

#include <cstdint>

#include "kea_lowbit.h"
#include "gemm_kernel.cuh"

namespace kea {

// ---- prepare: export codes -> panels --------------------------------------------------------------------------
// Within each 32-bit panel word the export codes (LSB first) are re-ordered so that the expansion is a byte-permute
// lookup: 1 bit - code i moves to bit 4 (i % 8) + i / 8, so (word >> j) & 0x11111111 holds codes 8 j .. 8 j + 7 one
// per nibble; 2 bits - field i moves to bits 4 (i % 8) + 2 (i / 8), so word & 0x33333333 holds fields 0-7 and
// (word >> 2) & 0x33333333 fields 8-15, one per nibble. A nibble is then a prmt selector into a 4-byte table.
KEA_DEVI uint32_t interleave_codes(uint32_t w, int wbits) {
    uint32_t out = 0;
    if (wbits == 1) {
#pragma unroll
        for (int i = 0; i < 32; ++i) out |= ((w >> i) & 1u) << (4 * (i & 7) + (i >> 3));
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) out |= ((w >> (2 * i)) & 3u) << (4 * (i & 7) + 2 * (i >> 3));
    }
    return out;
}

// Panel layout: [ceil(N/128) tiles][ceil(K/128) k-blocks][wbits sub-blocks][4 words][128 rows][4 bytes]. Sub-block s
// of k-block b of channel row 128 t + r covers k in [128 b + s * 128 / wbits, ... + 128 / wbits): the 16 export bytes
// of that row starting at byte 16 wbits b + 16 s (zero past the row end), read as four little-endian words whose
// codes are then interleaved (below), word j stored at (j * 128 + r) * 4 (word-major, so the kernel's per-row word
// loads hit distinct banks). One thread builds one row of one sub-block and checks its bytes: bits past k = K must be 0, and a 2-bit
// field must not be 0b11.
__global__ void __launch_bounds__(256) prepare_panels_kernel(const uint8_t *__restrict__ codes, int row_bytes, int wbits,
                                                             int N, int K, int kb_total, long long rows_total,
                                                             uint8_t *__restrict__ panels, uint32_t *err) {
    const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;   // (tile, k-block, sub-block, row)
    if (idx >= rows_total) return;
    const int r = (int)(idx % kPanelN);
    long long rest = idx / kPanelN;
    const int s = (int)(rest % wbits);
    rest /= wbits;
    const int b = (int)(rest % kb_total);
    const long long t = rest / kb_total;
    const long long n = t * kPanelN + r;
    const int byte0 = b * 16 * wbits + s * 16;
    const int per_byte = 8 / wbits;
    uint32_t bad = 0;
    uint32_t words[4] = {0, 0, 0, 0};
    if (n < N) {
        const uint8_t *src = codes + n * (long long)row_bytes;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int byte = byte0 + i;
            if (byte >= row_bytes) break;
            const uint32_t v = src[byte];
            const int valid = min(per_byte, K - byte * per_byte);  // codes of this byte that lie below K
            if (valid < per_byte && (v >> (valid * wbits)) != 0) bad |= KEA_DEVERR_TAIL_BITS;
            if (wbits == 2) {
                // a field is 0b11 when both of its bits are set: (v & (v >> 1)) has its even bit set
                const uint32_t both = v & (v >> 1) & 0x55u;
                const uint32_t live = valid >= 4 ? 0x55u : (0x55u & ((1u << (2 * valid)) - 1u));
                if (both & live) bad |= KEA_DEVERR_TERNARY_11;
            }
            words[i >> 2] |= v << (8 * (i & 3));
        }
    }
    uint32_t *dst = reinterpret_cast<uint32_t *>(panels + (idx - r) * 16);   // the sub-block's first byte
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[j * kPanelN + r] = interleave_codes(words[j], wbits);
    if (bad) report(err, bad);
}

// ---- residual INT8 quantizer ----------------------------------------------------------------------------------
struct QuantArgs {
    const float *x;
    long long xb, xt, xk;
    int t, M, K, parts, ldq;
    int8_t *q;
    long long q_stride;
    float *qs;
    long long qs_stride;
    const float *nw, *nb;
    float eps;
    int flags;
};

constexpr int kQuantThreads = 256;

KEA_DEVI float block_reduce(float v, bool use_max, float *scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xFFFFFFFFu, v, o);
        v = use_max ? fmaxf(v, u) : __fadd_rn(v, u);
    }
    __syncthreads();  // scratch may still be read by the previous reduction
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float r = scratch[0];
    for (int w = 1; w < kQuantThreads / 32; ++w) r = use_max ? fmaxf(r, scratch[w]) : __fadd_rn(r, scratch[w]);
    return r;
}

// One CTA per token row; the row lives in shared memory (K floats) while the parts are peeled off.
__global__ void __launch_bounds__(kQuantThreads) quantize_kernel(const QuantArgs a) {
    extern __shared__ float xrow[];
    __shared__ float scratch[kQuantThreads / 32];
    const int m = blockIdx.x;
    const float *x = a.x + (long long)(m / a.t) * a.xb + (long long)(m % a.t) * a.xt;
    grid_dependency_wait();
    for (int k = threadIdx.x; k < a.K; k += kQuantThreads) xrow[k] = x[(long long)k * a.xk];
    __syncthreads();
    if (a.nw) {
        float s = 0.f;
        for (int k = threadIdx.x; k < a.K; k += kQuantThreads) s = __fadd_rn(s, xrow[k]);
        const float mean = __fdiv_rn(block_reduce(s, false, scratch), (float)a.K);
        float v = 0.f;
        for (int k = threadIdx.x; k < a.K; k += kQuantThreads) {
            const float d = __fsub_rn(xrow[k], mean);
            v = __fmaf_rn(d, d, v);
        }
        const float var = __fdiv_rn(block_reduce(v, false, scratch), (float)a.K);
        const float inv = rsqrtf(__fadd_rn(var, a.eps));
        for (int k = threadIdx.x; k < a.K; k += kQuantThreads)
            xrow[k] = __fmaf_rn(__fmul_rn(__fsub_rn(xrow[k], mean), inv), a.nw[k], a.nb ? a.nb[k] : 0.f);
    }
    if (a.flags & 1) {
        for (int k = threadIdx.x; k < a.K; k += kQuantThreads) {
            const float v = xrow[k];
            xrow[k] = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
        }
    }
    __syncthreads();
    for (int p = 0; p < a.parts; ++p) {
        float amax = 0.f;
        for (int k = threadIdx.x; k < a.K; k += kQuantThreads) amax = fmaxf(amax, fabsf(xrow[k]));
        amax = block_reduce(amax, true, scratch);
        const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1.0e-30f);
        int8_t *q = a.q + p * a.q_stride + (long long)m * a.ldq;
        for (int k = threadIdx.x; k < a.ldq; k += kQuantThreads) {
            int8_t code = 0;
            if (k < a.K) {
                const float v = xrow[k];
                const float r = rintf(__fdiv_rn(v, scale));
                code = (int8_t)(int)r;
                xrow[k] = __fsub_rn(v, __fmul_rn(r, scale));
            }
            q[k] = code;
        }
        if (threadIdx.x == 0) a.qs[p * a.qs_stride + m] = scale;
        __syncthreads();
    }
    grid_launch_dependents();
}

}  // namespace kea
