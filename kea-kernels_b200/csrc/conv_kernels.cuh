// conv_kernels.cuh - the FastConformer convolution module's middle between its two pointwise GEMMs: GLU, padding
// mask and the depthwise convolution along time (BatchNorm folded into its weights), in one pass.
//
// In:  h FP32 [B][T][2C] (pw1's output, token-major as the GEMM writes it);
// out: y FP32 [B][T][C]  (token-major again: pw2's quantizer reads unit-stride rows);
//      g[b, t, c] = h[b, t, c] * sigmoid(h[b, t, C + c]), zero at t >= length[b] (padding) and outside [0, T);
//      y[b, t, c] = bias[c] + sum_j w[c, j] * g[b, t + j - KW / 2, c].
// Replaces the reference's glu_pad (Triton, src/kea_kernels/ternary/layer_fusions4.py:52-77) + the torch depthwise
// conv + batch norm, and the transposes around them. One thread per (clip, channel, chunk of kConvChunk frames)
// streams over its frames with the last KW GLU values in registers: consecutive threads take consecutive channels, so
// every load and store is a coalesced 128-byte warp access; each chunk recomputes its KW - 1 halo values.
// Memory-bound: 8 C bytes read and 4 C bytes written per frame (+ halo re-reads, L1/L2 hits).
#pragma once

#include "ptx.cuh"

namespace kea {

constexpr int kConvThreads = 256;
constexpr int kConvChunk = 16;   // output frames per thread
constexpr int kConvMaxKw = 31;   // odd kernel widths up to this

struct ConvArgs {
    const float *h;
    float *y;
    const float *w;              // [C][KW]
    const float *bias;           // [C] or null
    const int *lengths;          // [B] frames per clip, or null (every frame live)
    int B, T, C;
};

template <int KW>
__global__ void __launch_bounds__(kConvThreads) glu_depthwise_kernel(const ConvArgs a) {
    const int c = blockIdx.x * kConvThreads + threadIdx.x;
    const int b = blockIdx.z;
    const int t0 = blockIdx.y * kConvChunk;
    grid_dependency_wait();
    if (c >= a.C) return;
    constexpr int H = KW / 2;
    float w[KW];
#pragma unroll
    for (int j = 0; j < KW; ++j) w[j] = __ldg(a.w + (long long)c * KW + j);
    const float bias = a.bias ? __ldg(a.bias + c) : 0.f;
    const int live = a.lengths ? min(a.T, __ldg(a.lengths + b)) : a.T;
    const long long row2 = 2LL * a.C;
    const float *hb = a.h + (long long)b * a.T * row2;
    float *yb = a.y + (long long)b * a.T * a.C;
    float win[KW];   // win[j] = g at frame t - H + j for the output frame t being formed
    auto glu = [&](int t) -> float {
        if (t < 0 || t >= live) return 0.f;
        const float x = __ldg(hb + (long long)t * row2 + c), gate = __ldg(hb + (long long)t * row2 + a.C + c);
        return __fmul_rn(x, __frcp_rn(__fadd_rn(1.0f, expf(-gate))));
    };
#pragma unroll
    for (int j = 0; j < KW - 1; ++j) win[j + 1] = glu(t0 - H + j);
    const int t1 = min(a.T, t0 + kConvChunk);
#pragma unroll 4
    for (int t = t0; t < t1; ++t) {
#pragma unroll
        for (int j = 0; j < KW - 1; ++j) win[j] = win[j + 1];
        win[KW - 1] = glu(t + H);
        float acc = bias;
#pragma unroll
        for (int j = 0; j < KW; ++j) acc = __fmaf_rn(w[j], win[j], acc);
        yb[(long long)t * a.C + c] = acc;
    }
    grid_launch_dependents();
}

}  // namespace kea
