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

#include "aux_kernels.cuh"

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
        const float x = hb[(long long)t * row2 + c], gate = hb[(long long)t * row2 + a.C + c];
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

// ---- the same, with the next projection's quantizer fused in ---------------------------------------------------
// The conv module's output feeds only pw2, whose quantizer applies an input SiLU and peels off residual INT8 parts per
// frame row. A CTA here owns F whole frame rows (every channel of one clip, 4 channels a thread: C <= 1024), so each
// row's amax is a CTA reduction and the kernel writes pw2's INT8 parts and scales directly; the FP32 output is
// written only when asked for. Every value is computed with the operations, in the order, of glu_depthwise_kernel
// and then quantize_regs_kernel (GLU, the depthwise sum from the bias up, SiLU, scale = max(amax / 127, 1e-30),
// quantize4, residual), and amax is a maximum (order-free), so the parts and scales equal those two kernels' bit for
// bit. The F + KW - 1 frames of GLU values a CTA needs are loaded at once (16-byte loads, no serial dependence).
constexpr int kConvQThreads = 256;
constexpr int kConvQMaxC = 4 * kConvQThreads;

struct ConvQuantArgs {
    ConvArgs c;                  // y may be null
    int8_t *q;
    long long q_stride;
    int ldq;
    float *qs;
    long long qs_stride;
    int parts;
    int silu;
};

template <int KW, int F>
__global__ void __launch_bounds__(kConvQThreads) glu_depthwise_quant_kernel(const ConvQuantArgs a) {
    constexpr int H = KW / 2, W = F + KW - 1, NW = kConvQThreads / 32;
    __shared__ float red[3][F][NW];   // one slot per part: the per-row partial maxima of the CTA's warps
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int C = a.c.C, T = a.c.T;
    const int c0 = 4 * tid;
    const bool has = c0 < C;          // C % 4 == 0
    const int b = blockIdx.y, t0 = blockIdx.x * F;
    float w[4][KW], bias[4];
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
#pragma unroll
        for (int j = 0; j < KW; ++j) w[ch][j] = has ? __ldg(a.c.w + (long long)(c0 + ch) * KW + j) : 0.f;
        bias[ch] = has && a.c.bias ? __ldg(a.c.bias + c0 + ch) : 0.f;
    }
    grid_dependency_wait();
    const int live = a.c.lengths ? min(T, __ldg(a.c.lengths + b)) : T;
    const long long row2 = 2LL * C;
    const float *hb = a.c.h + (long long)b * T * row2;
    float4 xv[W], gv[W];
#pragma unroll
    for (int i = 0; i < W; ++i) {
        const int t = t0 - H + i;
        const bool in = has && t >= 0 && t < live;
        xv[i] = in ? *reinterpret_cast<const float4 *>(hb + (long long)t * row2 + c0) : make_float4(0.f, 0.f, 0.f, 0.f);
        gv[i] = in ? *reinterpret_cast<const float4 *>(hb + (long long)t * row2 + C + c0) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float g[W][4];   // GLU values; zero outside the clip's live frames (as glu_depthwise_kernel)
#pragma unroll
    for (int i = 0; i < W; ++i) {
        const int t = t0 - H + i;
        const bool in = t >= 0 && t < live;
        const float *xs = reinterpret_cast<const float *>(&xv[i]), *gs = reinterpret_cast<const float *>(&gv[i]);
#pragma unroll
        for (int ch = 0; ch < 4; ++ch)
            g[i][ch] = in ? __fmul_rn(xs[ch], __frcp_rn(__fadd_rn(1.0f, expf(-gs[ch])))) : 0.f;
    }
    float v[F][4];
#pragma unroll
    for (int f = 0; f < F; ++f) {
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
            float acc = bias[ch];
#pragma unroll
            for (int j = 0; j < KW; ++j) acc = __fmaf_rn(w[ch][j], g[f + j][ch], acc);
            v[f][ch] = acc;
        }
        if (a.c.y && has && t0 + f < T)
            *reinterpret_cast<float4 *>(a.c.y + ((long long)b * T + t0 + f) * C + c0) =
                make_float4(v[f][0], v[f][1], v[f][2], v[f][3]);
    }
    float amax[F];
#pragma unroll
    for (int f = 0; f < F; ++f) {
        amax[f] = 0.f;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
            if (a.silu) v[f][ch] = __fdiv_rn(v[f][ch], __fadd_rn(1.0f, expf(-v[f][ch])));
            if (has) amax[f] = fmaxf(amax[f], fabsf(v[f][ch]));
        }
    }
    for (int p = 0; p < a.parts; ++p) {
#pragma unroll
        for (int f = 0; f < F; ++f) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax[f] = fmaxf(amax[f], __shfl_xor_sync(0xFFFFFFFFu, amax[f], o));
            if (lane == 0) red[p][f][warp] = amax[f];
        }
        __syncthreads();
#pragma unroll
        for (int f = 0; f < F; ++f) {
            float r = red[p][f][0];
#pragma unroll
            for (int k = 1; k < NW; ++k) r = fmaxf(r, red[p][f][k]);
            const float scale = fmaxf(__fdiv_rn(r, 127.0f), 1.0e-30f);
            const float rcp = __frcp_rn(scale);
            const int t = t0 + f;
            const long long m = (long long)b * T + t;
            float codes[4];
            const uint32_t word = quantize4(v[f], scale, rcp, codes);
            float next = 0.f;
#pragma unroll
            for (int ch = 0; ch < 4; ++ch) {
                v[f][ch] = __fsub_rn(v[f][ch], __fmul_rn(codes[ch], scale));
                if (has) next = fmaxf(next, fabsf(v[f][ch]));
            }
            amax[f] = next;
            if (t < T) {
                uint32_t *q = reinterpret_cast<uint32_t *>(a.q + p * a.q_stride + m * a.ldq);
                if (has) q[tid] = word;
                for (int i = C / 4 + tid; i < a.ldq / 4; i += kConvQThreads) q[i] = 0u;   // padding columns
                if (tid == 0) a.qs[p * a.qs_stride + m] = scale;
            }
        }
    }
    grid_launch_dependents();
}

}  // namespace kea
