// quant_common.cuh - the residual INT8 quantizer's per-value arithmetic, shared by the quantizer kernels
// (aux_kernels.cuh), the conv kernel's fused quantizer (conv_kernels.cuh) and the GEMM kernel's fused prologue
// quantizer (gemm_kernel.cuh), so every path rounds the same way.
#pragma once

#include <cstdint>

#include "ptx.cuh"

namespace kea {

// rint(v / s) with the IEEE round-to-nearest quotient, without a division on the common path. Here |v| <= 127 s
// (s is the part's amax / 127, or larger), so |v / s| <= 127 + 1e-4, and q = RN(v * RN(1 / s)) differs from v / s
// by at most 2 * 2^-24 * 127 < 1.6e-5 while the IEEE quotient differs from v / s by at most 7.6e-6: the two round to
// the same integer unless a half-integer lies within 2.4e-5 of q. Values within 1e-4 of a half-integer (and anything
// non-finite or out of range) take the exact division.
KEA_DEVI float round_quotient(float v, float s, float inv) {
    const float q = __fmul_rn(v, inv);
    const float f = fabsf(q - truncf(q));
    if (fabsf(f - 0.5f) > 1.0e-4f && fabsf(q) < 128.0f) return rintf(q);
    return rintf(__fdiv_rn(v, s));
}

// Four codes rint(e[j] / s) (the IEEE quotient, as round_quotient) packed little-endian into a word; r[j] gets the
// codes as floats. Branch-free on the common path: the four products e[j] * RN(1 / s) are rounded together and one
// flag records whether any lies within 1e-4 of a half-integer (or is not a number); only then are the four redone
// with the exact division.
KEA_DEVI uint32_t quantize4(const float *e, float s, float inv, float (&r)[4]) {
    bool odd = false;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float t = __fmul_rn(e[j], inv);
        r[j] = rintf(t);
        odd |= !(fabsf(__fsub_rn(t, r[j])) < 0.4999f);
    }
    if (odd) {
#pragma unroll
        for (int j = 0; j < 4; ++j) r[j] = rintf(__fdiv_rn(e[j], s));
    }
    const int b0 = __float2int_rn(r[0]), b1 = __float2int_rn(r[1]), b2 = __float2int_rn(r[2]), b3 = __float2int_rn(r[3]);
    return __byte_perm(__byte_perm(b0, b1, 0x0040), __byte_perm(b2, b3, 0x0040), 0x5410);
}

// ---- one warp, one row (K <= 1024): the GEMM's fused prologue quantizer ----------------------------------------
// The arithmetic of quantize_regs_kernel at 32 threads per row, step for step: lane l holds the float4 chunks at
// columns (c * 32 + l) * 4, c < 8 (zeros past K); sums over a lane's chunks in order, then the xor-shuffle tree of
// group_reduce; the LayerNorm as layer_norm_regs; one part. The affine parameters may live in shared memory.
constexpr int kRowChunks = 8;

KEA_DEVI float warp_sum_tree(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}
KEA_DEVI float warp_max_tree(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

KEA_DEVI void warp_layer_norm(float4 (&v)[kRowChunks], int K, int lane, const float *w, const float *b, float eps) {
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c) s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v[c].x), v[c].y), v[c].z), v[c].w);
    const float mean = __fdiv_rn(warp_sum_tree(s), (float)K);
    float var = 0.f;
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c) {
        if (4 * (c * 32 + lane) < K) {
            const float d0 = __fsub_rn(v[c].x, mean), d1 = __fsub_rn(v[c].y, mean);
            const float d2 = __fsub_rn(v[c].z, mean), d3 = __fsub_rn(v[c].w, mean);
            var = __fmaf_rn(d3, d3, __fmaf_rn(d2, d2, __fmaf_rn(d1, d1, __fmaf_rn(d0, d0, var))));
        }
    }
    const float inv = rsqrtf(__fadd_rn(__fdiv_rn(warp_sum_tree(var), (float)K), eps));
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c) {
        const int i = c * 32 + lane;
        if (4 * i < K) {
            const float4 ww = reinterpret_cast<const float4 *>(w)[i];
            const float4 bb = b ? reinterpret_cast<const float4 *>(b)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            v[c].x = __fmaf_rn(__fmul_rn(__fsub_rn(v[c].x, mean), inv), ww.x, bb.x);
            v[c].y = __fmaf_rn(__fmul_rn(__fsub_rn(v[c].y, mean), inv), ww.y, bb.y);
            v[c].z = __fmaf_rn(__fmul_rn(__fsub_rn(v[c].z, mean), inv), ww.z, bb.z);
            v[c].w = __fmaf_rn(__fmul_rn(__fsub_rn(v[c].w, mean), inv), ww.w, bb.w);
        }
    }
}

// Input SiLU (every chunk, as the quantizer kernel), the row's amax, one part: returns the scale and the code words
// of the lane's chunks (words[c] for 4 * (c * 32 + lane) < K).
KEA_DEVI float warp_quantize_row(float4 (&v)[kRowChunks], int K, int lane, bool silu, uint32_t (&words)[kRowChunks]) {
    if (silu) {
#pragma unroll
        for (int c = 0; c < kRowChunks; ++c) {
            v[c].x = __fdiv_rn(v[c].x, __fadd_rn(1.0f, expf(-v[c].x)));
            v[c].y = __fdiv_rn(v[c].y, __fadd_rn(1.0f, expf(-v[c].y)));
            v[c].z = __fdiv_rn(v[c].z, __fadd_rn(1.0f, expf(-v[c].z)));
            v[c].w = __fdiv_rn(v[c].w, __fadd_rn(1.0f, expf(-v[c].w)));
        }
    }
    float amax = 0.f;
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c)
        if (4 * (c * 32 + lane) < K)
            amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[c].x), fabsf(v[c].y)), fmaxf(fabsf(v[c].z), fabsf(v[c].w))));
    amax = warp_max_tree(amax);
    const float scale = fmaxf(__fdiv_rn(amax, 127.0f), 1.0e-30f);
    const float rcp = __frcp_rn(scale);
#pragma unroll
    for (int c = 0; c < kRowChunks; ++c) {
        float r[4];
        words[c] = quantize4(reinterpret_cast<const float *>(&v[c]), scale, rcp, r);
    }
    return scale;
}

}  // namespace kea
