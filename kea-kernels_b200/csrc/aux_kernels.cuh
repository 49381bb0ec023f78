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
    // optional LayerNorm before everything else (a layer's output norm), its result written to `normed` [M][ldn]
    const float *pnw, *pnb;
    float peps;
    float *normed;
    long long ldn;
};

constexpr int kQuantThreads = 256;

// Sum / max over the `tpr` threads of each row group (tpr = 32, 64, 128 or 256; groups are whole warps), in a fixed
// order, so every thread of the group gets the same value. Every thread of the CTA must call it.
KEA_DEVI float group_reduce(float v, bool use_max, int tpr, float *scratch) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xFFFFFFFFu, v, o);
        v = use_max ? fmaxf(v, u) : __fadd_rn(v, u);
    }
    if (tpr == 32) return v;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wpr = tpr >> 5;
    __syncthreads();   // scratch may still be read by the previous reduction
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    const int w0 = warp - warp % wpr;
    float r = scratch[w0];
    for (int w = 1; w < wpr; ++w) r = use_max ? fmaxf(r, scratch[w0 + w]) : __fadd_rn(r, scratch[w0 + w]);
    return r;
}

// group_reduce with a scratch slot of its own (kQuantThreads / 32 floats) per reduction of the kernel, so no
// barrier is needed before the slot is written (no earlier reduction can still be reading it). Same order of
// operations as group_reduce, so the same result bit for bit.
KEA_DEVI float group_reduce_slot(float v, bool use_max, int tpr, float *slot) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float u = __shfl_xor_sync(0xFFFFFFFFu, v, o);
        v = use_max ? fmaxf(v, u) : __fadd_rn(v, u);
    }
    if (tpr == 32) return v;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, wpr = tpr >> 5;
    if (lane == 0) slot[warp] = v;
    __syncthreads();
    const int w0 = warp - warp % wpr;
    float r = slot[w0];
    for (int w = 1; w < wpr; ++w) r = use_max ? fmaxf(r, slot[w0 + w]) : __fadd_rn(r, slot[w0 + w]);
    return r;
}

// The affine parameters of a LayerNorm for the chunks a thread holds (zeros past K or without a bias): loaded before
// the kernel waits for the previous grid, since they do not depend on it.
template <int C>
KEA_DEVI void load_affine(const float *nw, const float *nb, int K, int tpr, int gt, float4 (&w)[C], float4 (&b)[C]) {
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int i = c * tpr + gt;
        const bool in = nw && 4 * i < K;
        w[c] = in ? __ldg(reinterpret_cast<const float4 *>(nw) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
        b[c] = in && nb ? __ldg(reinterpret_cast<const float4 *>(nb) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
}

// LayerNorm of the row group's K values held as float4 chunks at (c * tpr + gt) * 4 (layout of
// quantize_regs_kernel): mean, then the centred variance (two group reductions in a fixed order, in scratch slots
// `slots` and `slots` + kQuantThreads / 32), then (v - mean) * rsqrt(var + eps) * w + b chunk by chunk, with w / b
// from `pw` / `pb` when PRE (loaded early by load_affine), else read here. Chunks past K stay as they are.
template <int C, bool PRE>
KEA_DEVI void layer_norm_regs(float4 (&v)[C], int K, int tpr, int gt, float *slots, const float *nw,
                              const float *nb, float eps, const float4 (&pw)[C], const float4 (&pb)[C]) {
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[c].x), v[c].y), v[c].z), v[c].w);
    const float mean = __fdiv_rn(group_reduce_slot(s, false, tpr, slots), (float)K);
    float var = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
        if (4 * (c * tpr + gt) < K) {
            const float d0 = __fsub_rn(v[c].x, mean), d1 = __fsub_rn(v[c].y, mean);
            const float d2 = __fsub_rn(v[c].z, mean), d3 = __fsub_rn(v[c].w, mean);
            var = __fmaf_rn(d3, d3, __fmaf_rn(d2, d2, __fmaf_rn(d1, d1, __fmaf_rn(d0, d0, var))));
        }
    }
    const float inv = rsqrtf(__fadd_rn(__fdiv_rn(group_reduce_slot(var, false, tpr, slots + kQuantThreads / 32), (float)K), eps));
    // the affine parameters are read here, chunk by chunk, not held for the whole row (registers)
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int i = c * tpr + gt;
        if (4 * i < K) {
            const float4 w = PRE ? pw[c] : __ldg(reinterpret_cast<const float4 *>(nw) + i);
            const float4 b = PRE ? pb[c] : (nb ? __ldg(reinterpret_cast<const float4 *>(nb) + i) : make_float4(0.f, 0.f, 0.f, 0.f));
            v[c].x = __fmaf_rn(__fmul_rn(__fsub_rn(v[c].x, mean), inv), w.x, b.x);
            v[c].y = __fmaf_rn(__fmul_rn(__fsub_rn(v[c].y, mean), inv), w.y, b.y);
            v[c].z = __fmaf_rn(__fmul_rn(__fsub_rn(v[c].z, mean), inv), w.z, b.z);
            v[c].w = __fmaf_rn(__fmul_rn(__fsub_rn(v[c].w, mean), inv), w.w, b.w);
        }
    }
}

// The register-resident quantizer for unit-stride rows (xk == 1, K a multiple of 4, 16-byte aligned rows): `tpr`
// threads per row (32 .. 256, 256 / tpr rows per CTA), each holding VPT = K / tpr (rounded up to 4) values as float4
// chunks at (c * tpr + thread) * 4, so every load and store is a coalesced 16-byte vector. LayerNorm takes two
// group reductions (mean, then the centred variance), each part one (amax); nothing goes through shared memory but
// the reductions' partials. This is the path of every encoder call site; other layouts take quantize_kernel.
template <int VPT>
__global__ void __launch_bounds__(kQuantThreads) quantize_regs_kernel(const QuantArgs a, int tpr) {
    // one scratch slot per reduction: pre-norm mean / variance, norm mean / variance, one amax per part
    constexpr int kSlot = kQuantThreads / 32;
    __shared__ float scratch[7 * kSlot];
    constexpr int C = VPT / 4;
    // up to 4 chunks a thread the LayerNorms' affine parameters are held in registers, loaded before the wait
    constexpr bool PRE = C <= 4;
    const int rows = kQuantThreads / tpr;
    const int g = threadIdx.x / tpr, gt = threadIdx.x % tpr;
    const int m = blockIdx.x * rows + g;
    const bool live = m < a.M;
    const int K = a.K;
    float4 v[C];
    float4 pw[C], pb[C], nw[C], nb[C];   // unused (and dropped by the compiler) unless PRE
    if (PRE) {
        load_affine<C>(a.pnw, a.pnb, K, tpr, gt, pw, pb);
        load_affine<C>(a.nw, a.nb, K, tpr, gt, nw, nb);
    }
    grid_dependency_wait();
    // the next kernel may launch now: it loads its static operands, then waits for this grid to complete
    grid_launch_dependents();
    const float4 *src = reinterpret_cast<const float4 *>(
        a.x + (live ? (long long)(m / a.t) * a.xb + (long long)(m % a.t) * a.xt : 0LL));
#pragma unroll
    for (int c = 0; c < C; ++c) {
        const int i = c * tpr + gt;
        v[c] = (live && 4 * i < K) ? src[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (a.pnw) {
        layer_norm_regs<C, PRE>(v, K, tpr, gt, scratch, a.pnw, a.pnb, a.peps, pw, pb);
        if (live) {
            float4 *dst = reinterpret_cast<float4 *>(a.normed + (long long)m * a.ldn);
#pragma unroll
            for (int c = 0; c < C; ++c) {
                const int i = c * tpr + gt;
                if (4 * i < K) dst[i] = v[c];
            }
        }
    }
    if (a.nw)
        layer_norm_regs<C, PRE>(v, K, tpr, gt, scratch + 2 * kSlot, a.nw, a.nb, a.eps, nw, nb);
    if (a.flags & 1) {
#pragma unroll
        for (int c = 0; c < C; ++c) {
            v[c].x = __fdiv_rn(v[c].x, __fadd_rn(1.0f, expf(-v[c].x)));
            v[c].y = __fdiv_rn(v[c].y, __fadd_rn(1.0f, expf(-v[c].y)));
            v[c].z = __fdiv_rn(v[c].z, __fadd_rn(1.0f, expf(-v[c].z)));
            v[c].w = __fdiv_rn(v[c].w, __fadd_rn(1.0f, expf(-v[c].w)));
        }
    }
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c)
        if (4 * (c * tpr + gt) < K)
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[c].x), fabsf(v[c].y)), fmaxf(fabsf(v[c].z), fabsf(v[c].w))));
    for (int p = 0; p < a.parts; ++p) {
        amax = group_reduce_slot(amax, true, tpr, scratch + (4 + p) * kSlot);
        const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1.0e-30f);
        const float rcp = __frcp_rn(scale);
        float next = 0.f;   // the residual's amax: the next part's scale
        uint32_t *q = reinterpret_cast<uint32_t *>(a.q + p * a.q_stride + (long long)m * a.ldq);
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const int i = c * tpr + gt;
            if (4 * i < K) {
                float *e = reinterpret_cast<float *>(&v[c]);
                float r[4];
                const uint32_t word = quantize4(e, scale, rcp, r);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    e[j] = __fsub_rn(e[j], __fmul_rn(r[j], scale));
                    next = fmaxf(next, fabsf(e[j]));
                }
                if (live) q[i] = word;
            }
        }
        if (live) {
            for (int i = K / 4 + gt; i < a.ldq / 4; i += tpr) q[i] = 0u;   // padding columns
            if (gt == 0) a.qs[p * a.qs_stride + m] = scale;
        }
        amax = next;
    }
    grid_launch_dependents();
}

// `tpr` threads per token row (a power of two from 32 to 256; 256 / tpr rows per CTA): the host picks fewer threads
// per row when there are many rows (bandwidth) and more when there are few (latency). The CTA stages its rows in
// shared memory with loads whose consecutive threads read consecutive addresses: 16-byte vectors along k when the
// row stride xk is 1, consecutive rows of one column in the [B, K, T] conv layout (xt == 1). Each row group then
// normalizes (optional LayerNorm, input SiLU) and peels off the parts with group reductions; codes leave as 32-bit
// words (four per word), the padding columns k .. ldq - 1 as zeros.
__global__ void __launch_bounds__(kQuantThreads) quantize_kernel(const QuantArgs a, int tpr) {
    extern __shared__ float xrows[];
    __shared__ const float *bases[kQuantThreads / 32];
    __shared__ float scratch[kQuantThreads / 32];
    const int rows = kQuantThreads / tpr;
    const int g = threadIdx.x / tpr, gt = threadIdx.x % tpr;    // row group, thread within the group
    const int m0 = blockIdx.x * rows;
    const int nrows = min(rows, a.M - m0);
    const int K = a.K;
    if (threadIdx.x < nrows) {
        const int m = m0 + threadIdx.x;
        bases[threadIdx.x] = a.x + (long long)(m / a.t) * a.xb + (long long)(m % a.t) * a.xt;
    }
    grid_dependency_wait();
    // the next kernel may launch now: it loads its static operands, then waits for this grid to complete
    grid_launch_dependents();
    __syncthreads();
    if (a.xk == 1) {
        if (g < nrows) {
            const float *src = bases[g];
            float *dst = xrows + g * K;
            if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0 && (K & 3) == 0) {
                const float4 *s4 = reinterpret_cast<const float4 *>(src);
                float4 *d4 = reinterpret_cast<float4 *>(dst);
#pragma unroll 4
                for (int i = gt; i < K / 4; i += tpr) d4[i] = s4[i];
            } else {
#pragma unroll 4
                for (int k = gt; k < K; k += tpr) dst[k] = src[k];
            }
        }
    } else {
        const int per = kQuantThreads / nrows;
        const int r = threadIdx.x % nrows, k0 = threadIdx.x / nrows;
        if (k0 < per) {
            const float *src = bases[r];
            float *dst = xrows + r * K;
#pragma unroll 4
            for (int k = k0; k < K; k += per) dst[k] = src[(long long)k * a.xk];
        }
    }
    __syncthreads();
    const bool live = g < nrows;
    const int m = m0 + g;
    float *row = xrows + (live ? g : 0) * K;
    if (a.nw) {
        float s = 0.f;
        if (live)
            for (int k = gt; k < K; k += tpr) s = __fadd_rn(s, row[k]);
        const float mean = __fdiv_rn(group_reduce(s, false, tpr, scratch), (float)K);
        float v = 0.f;
        if (live)
            for (int k = gt; k < K; k += tpr) {
                const float d = __fsub_rn(row[k], mean);
                v = __fmaf_rn(d, d, v);
            }
        const float var = __fdiv_rn(group_reduce(v, false, tpr, scratch), (float)K);
        const float inv = rsqrtf(__fadd_rn(var, a.eps));
        if (live)
            for (int k = gt; k < K; k += tpr)
                row[k] = __fmaf_rn(__fmul_rn(__fsub_rn(row[k], mean), inv), a.nw[k], a.nb ? a.nb[k] : 0.f);
    }
    if ((a.flags & 1) && live) {
        for (int k = gt; k < K; k += tpr) {
            const float v = row[k];
            row[k] = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
        }
    }
    __syncthreads();
    for (int p = 0; p < a.parts; ++p) {
        float amax = 0.f;
        if (live)
            for (int k = gt; k < K; k += tpr) amax = fmaxf(amax, fabsf(row[k]));
        amax = group_reduce(amax, true, tpr, scratch);
        const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1.0e-30f);
        const float inv = __frcp_rn(scale);
        if (live) {
            uint32_t *q = reinterpret_cast<uint32_t *>(a.q + p * a.q_stride + (long long)m * a.ldq);
            const bool vec = (K & 3) == 0;   // whole 16-byte groups of the row: one shared-memory vector each
            for (int w = gt; w < a.ldq / 4; w += tpr) {   // ldq is a multiple of 4: whole words
                uint32_t word = 0;
                if (vec && 4 * w < K) {
                    float4 v4 = reinterpret_cast<const float4 *>(row)[w];
                    float *v = reinterpret_cast<float *>(&v4);
                    float r[4];
                    word = quantize4(v, scale, inv, r);
#pragma unroll
                    for (int j = 0; j < 4; ++j) v[j] = __fsub_rn(v[j], __fmul_rn(r[j], scale));
                    reinterpret_cast<float4 *>(row)[w] = v4;
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int k = 4 * w + j;
                        if (k < K) {
                            const float v = row[k];
                            const float r = round_quotient(v, scale, inv);
                            word |= ((uint32_t)(int)r & 0xFFu) << (8 * j);
                            row[k] = __fsub_rn(v, __fmul_rn(r, scale));
                        }
                    }
                }
                q[w] = word;
            }
            if (gt == 0) a.qs[p * a.qs_stride + m] = scale;
        }
        __syncthreads();
    }
    grid_launch_dependents();
}

}  // namespace kea
