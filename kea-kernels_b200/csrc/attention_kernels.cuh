// attention_kernels.cuh - the FastConformer's relative-position self-attention, FP32, in one kernel.
//
// In:  qkv FP32 [B][T][3][H][DK] (the fused QKV GEMM's output rows), pos FP32 [2T - 1][H][DK] (linear_pos applied to
//      the sinusoidal table of relative positions T - 1 .. -(T - 1)), bias_u / bias_v FP32 [H][DK], optional key
//      lengths [B];
// out: ctx FP32 [B][T][H][DK] (token-major: the out projection's input rows).
//   score[i, j] = ((q_i + u) . k_j + (q_i + v) . pos[j + T - 1 - i]) * scale,   keys j >= length masked,
//   ctx_i = softmax_j(score[i, :]) . v.
// The second term is Transformer-XL's shifted position score (rel_shift of (q + v) . pos^T). This replaces the
// reference's fused relative attention (src/kea_kernels/ternary/fused_kernels.py, relative_attention) and the
// torch sequence around it (bias adds, permutes, three matmuls, the shift, softmax, the transpose back).
//
// One CTA = 32 queries of one (clip, head); key blocks of 32 stream through shared memory with an online softmax
// (running max and sum per query, rescaled accumulators), so no T x T matrix is ever written. Per key block the CTA
// stages K, V and the band of 63 position rows that the 32 x 32 score tile touches (relative offsets j - i in
// [j0 - i0 - 31, j0 - i0 + 31]). 128 threads: a thread scores 2 queries x 4 consecutive keys (ac and bd dot products
// over DK from shared memory, 16-byte vectors; the 2 x 4 block needs only 5 band rows), and accumulates 2 queries x
// DK / 8 output columns (16-byte chunks c, c + 8, ...). The 8 lanes of a shared-memory phase read K and band rows
// four apart, so those tiles store 16-byte chunk c of row r at c ^ ((r / 4) % 8): conflict-free. FP32 FMAs
// throughout; the softmax uses expf and the final division is IEEE.
//
// KG = 2 (small grids: one clip gives only 32 CTAs) doubles the CTA to two 128-thread groups that take alternate key
// blocks, each with its own K / V / band / probability tiles and online-softmax state; the two states are merged at
// the end (max, rescaled sums), halving the chain of key blocks each CTA walks.
#pragma once

#include "ptx.cuh"

namespace kea {

constexpr int kAttnThreads = 128;
constexpr int kAttnQ = 32, kAttnK = 32;
constexpr int kAttnBand = kAttnQ + kAttnK - 1;

struct RelAttnArgs {
    const float *qkv;
    const float *pos;
    const float *bias_u, *bias_v;
    const int *lengths;          // [B] or null
    float *ctx;
    int B, T, H;
    float scale;
};

// Shared memory floats for head width DK: Qu, Qv (rows padded by 4), then per key group a V tile (padded), K and the
// position band (swizzled) and the probability tile.
template <int DK>
__host__ __device__ constexpr int attn_group_floats() {
    return kAttnK * (DK + 4) + (kAttnK + kAttnBand) * DK + kAttnQ * (kAttnK + 1);
}
template <int DK, int KG>
__host__ __device__ constexpr int attn_smem_floats() {
    return 2 * kAttnQ * (DK + 4) + KG * attn_group_floats<DK>();
}
// float offset of 16-byte chunk c4 of row r in a swizzled tile of DK-float rows
template <int DK>
KEA_DEVI int swz(int r, int c4) { return r * DK + 4 * (c4 ^ ((r >> 2) & 7)); }

template <int DK, int KG>
__global__ void __launch_bounds__(kAttnThreads * KG) rel_attention_kernel(const RelAttnArgs a) {
    extern __shared__ __align__(16) float asmem[];
    static_assert(DK % 32 == 0, "head width: a multiple of 32 (eight 16-byte chunks for the swizzle)");
    constexpr int LD = DK + 4;   // padded row: 16-byte aligned, rows start on different banks
    const int g = threadIdx.x / kAttnThreads, tid = threadIdx.x % kAttnThreads;   // key group, thread within it
    float *Qu = asmem, *Qv = Qu + kAttnQ * LD;
    float *Vs = Qv + kAttnQ * LD + g * attn_group_floats<DK>();
    float *Ks = Vs + kAttnK * LD, *Ps = Ks + kAttnK * DK, *Pr = Ps + kAttnBand * DK;   // Pr: [kAttnQ][kAttnK + 1]
    const int i0 = blockIdx.x * kAttnQ, h = blockIdx.y, b = blockIdx.z;
    const int T = a.T, H = a.H;
    const long long row3 = 3LL * H * DK;   // floats per token row of qkv
    const float *qkv_b = a.qkv + (long long)b * T * row3;
    const int live = a.lengths ? min(T, __ldg(a.lengths + b)) : T;
    grid_dependency_wait();

    constexpr int V4 = DK / 4;   // float4 per head row
    // queries (+ both position biases)
    for (int e = threadIdx.x; e < kAttnQ * V4; e += kAttnThreads * KG) {
        const int r = e / V4, c4 = e - r * V4, i = i0 + r;
        float4 q = make_float4(0.f, 0.f, 0.f, 0.f);
        if (i < T) q = reinterpret_cast<const float4 *>(qkv_b + (long long)i * row3 + (long long)h * DK)[c4];
        const float4 u = __ldg(reinterpret_cast<const float4 *>(a.bias_u + h * DK) + c4);
        const float4 v = __ldg(reinterpret_cast<const float4 *>(a.bias_v + h * DK) + c4);
        *reinterpret_cast<float4 *>(Qu + r * LD + 4 * c4) =
            make_float4(__fadd_rn(q.x, u.x), __fadd_rn(q.y, u.y), __fadd_rn(q.z, u.z), __fadd_rn(q.w, u.w));
        *reinterpret_cast<float4 *>(Qv + r * LD + 4 * c4) =
            make_float4(__fadd_rn(q.x, v.x), __fadd_rn(q.y, v.y), __fadd_rn(q.z, v.z), __fadd_rn(q.w, v.w));
    }

    // score layout: thread -> queries qi0, qi0 + 1 and keys kj0 .. kj0 + 3 of the 32 x 32 tile
    const int qi0 = 2 * (tid >> 3), kj0 = 4 * (tid & 7);
    // output layout: thread -> queries qi0, qi0 + 1 and the 16-byte chunks (tid % 8) + 8 m of the head row
    constexpr int OC = DK / 8;
    const int oc4 = tid & 7;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    float o[2][OC];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < OC; ++c) o[r][c] = 0.f;

    // group g takes key blocks g, g + KG, ...; every thread passes every barrier (a group without a block idles)
    const int trips = ((live + kAttnK - 1) / kAttnK + KG - 1) / KG;
    for (int trip = 0; trip < trips; ++trip) {
        const int j0 = (trip * KG + g) * kAttnK;
        const bool act = j0 < live;
        __syncthreads();   // the previous block's K / V / band / probabilities are consumed
        if (act)
        for (int e = tid; e < kAttnK * V4; e += kAttnThreads) {
            const int r = e / V4, c4 = e - r * V4, j = j0 + r;
            float4 kk = make_float4(0.f, 0.f, 0.f, 0.f), vv = kk;
            if (j < T) {
                const float *src = qkv_b + (long long)j * row3 + (long long)h * DK;
                kk = reinterpret_cast<const float4 *>(src + (long long)H * DK)[c4];
                vv = reinterpret_cast<const float4 *>(src + 2LL * H * DK)[c4];
            }
            *reinterpret_cast<float4 *>(Ks + swz<DK>(r, c4)) = kk;
            *reinterpret_cast<float4 *>(Vs + r * LD + 4 * c4) = vv;
        }
        // band row s <-> relative offset (j - i) = j0 - i0 - (kAttnQ - 1) + s <-> pos row offset + T - 1
        const int rel0 = j0 - i0 - (kAttnQ - 1);
        if (act)
        for (int e = tid; e < kAttnBand * V4; e += kAttnThreads) {
            const int s = e / V4, c4 = e - s * V4, pr = rel0 + s + T - 1;
            float4 pp = make_float4(0.f, 0.f, 0.f, 0.f);
            if (pr >= 0 && pr < 2 * T - 1)
                pp = reinterpret_cast<const float4 *>(a.pos + ((long long)pr * H + h) * DK)[c4];
            *reinterpret_cast<float4 *>(Ps + swz<DK>(s, c4)) = pp;
        }
        __syncthreads();
        if (!act) {   // this group has no block in this trip: only the barriers
            __syncthreads();
            continue;
        }

        // scores: ac = Qu_i . K_j, bd = Qv_i . P_(j - i), for 2 x 4 (i, j)
        float ac[2][4], bd[2][4];
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
            for (int c = 0; c < 4; ++c) ac[r][c] = bd[r][c] = 0.f;
        // band index of (qi0 + r, kj0 + c) is (kj0 + c) - (qi0 + r) + kAttnQ - 1: five rows cover the 2 x 4 block
        const int sb = kj0 - qi0 - 1 + (kAttnQ - 1);
#pragma unroll 4
        for (int d4 = 0; d4 < V4; ++d4) {
            float4 qu[2], qv[2], kv[4], pv[5];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                qu[r] = *reinterpret_cast<const float4 *>(Qu + (qi0 + r) * LD + 4 * d4);
                qv[r] = *reinterpret_cast<const float4 *>(Qv + (qi0 + r) * LD + 4 * d4);
            }
#pragma unroll
            for (int c = 0; c < 4; ++c) kv[c] = *reinterpret_cast<const float4 *>(Ks + swz<DK>(kj0 + c, d4));
#pragma unroll
            for (int s = 0; s < 5; ++s) pv[s] = *reinterpret_cast<const float4 *>(Ps + swz<DK>(sb + s, d4));
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    float x = ac[r][c];
                    x = __fmaf_rn(qu[r].x, kv[c].x, x);
                    x = __fmaf_rn(qu[r].y, kv[c].y, x);
                    x = __fmaf_rn(qu[r].z, kv[c].z, x);
                    ac[r][c] = __fmaf_rn(qu[r].w, kv[c].w, x);
                    const float4 p = pv[c - r + 1];   // band row (kj0 + c) - (qi0 + r) + 31 - sb
                    float y = bd[r][c];
                    y = __fmaf_rn(qv[r].x, p.x, y);
                    y = __fmaf_rn(qv[r].y, p.y, y);
                    y = __fmaf_rn(qv[r].z, p.z, y);
                    bd[r][c] = __fmaf_rn(qv[r].w, p.w, y);
                }
        }
        // online softmax over this block's keys (a query row's 32 scores live in 8 consecutive lanes)
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            float s[4], mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                s[c] = (j0 + kj0 + c < live) ? __fmul_rn(__fadd_rn(ac[r][c], bd[r][c]), a.scale) : -INFINITY;
                mx = fmaxf(mx, s[c]);
            }
#pragma unroll
            for (int w = 1; w < 8; w <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, w));
            const float m_new = fmaxf(m_run[r], mx);   // finite: key j0 < live is in every block processed
            const float corr = expf(m_run[r] - m_new);
            float sum = 0.f;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                s[c] = expf(s[c] - m_new);
                sum += s[c];
                Pr[(qi0 + r) * (kAttnK + 1) + kj0 + c] = s[c];
            }
#pragma unroll
            for (int w = 1; w < 8; w <<= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, w);
            l_run[r] = __fmaf_rn(l_run[r], corr, sum);
            m_run[r] = m_new;
#pragma unroll
            for (int c = 0; c < OC; ++c) o[r][c] = __fmul_rn(o[r][c], corr);
        }
        __syncthreads();
        // o += P . V for 2 queries x OC columns
#pragma unroll 4
        for (int j = 0; j < kAttnK; ++j) {
            const float p0 = Pr[qi0 * (kAttnK + 1) + j], p1 = Pr[(qi0 + 1) * (kAttnK + 1) + j];
#pragma unroll
            for (int c4 = 0; c4 < OC / 4; ++c4) {
                const float4 vv = *reinterpret_cast<const float4 *>(Vs + j * LD + 4 * (oc4 + 8 * c4));
                o[0][4 * c4] = __fmaf_rn(p0, vv.x, o[0][4 * c4]);
                o[0][4 * c4 + 1] = __fmaf_rn(p0, vv.y, o[0][4 * c4 + 1]);
                o[0][4 * c4 + 2] = __fmaf_rn(p0, vv.z, o[0][4 * c4 + 2]);
                o[0][4 * c4 + 3] = __fmaf_rn(p0, vv.w, o[0][4 * c4 + 3]);
                o[1][4 * c4] = __fmaf_rn(p1, vv.x, o[1][4 * c4]);
                o[1][4 * c4 + 1] = __fmaf_rn(p1, vv.y, o[1][4 * c4 + 1]);
                o[1][4 * c4 + 2] = __fmaf_rn(p1, vv.z, o[1][4 * c4 + 2]);
                o[1][4 * c4 + 3] = __fmaf_rn(p1, vv.w, o[1][4 * c4 + 3]);
            }
        }
    }
    if constexpr (KG > 1) {   // merge group 1's state into group 0's (group 1's tiles hold it: [kAttnQ][DK + 4])
        __syncthreads();
        float *cm = asmem + 2 * kAttnQ * LD + attn_group_floats<DK>();
        if (g == 1) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                float *row = cm + (qi0 + r) * LD;
#pragma unroll
                for (int c4 = 0; c4 < OC / 4; ++c4)
                    *reinterpret_cast<float4 *>(row + 4 * (oc4 + 8 * c4)) =
                        make_float4(o[r][4 * c4], o[r][4 * c4 + 1], o[r][4 * c4 + 2], o[r][4 * c4 + 3]);
                if (oc4 == 0) {
                    row[DK] = m_run[r];
                    row[DK + 1] = l_run[r];
                }
            }
        }
        __syncthreads();
        if (g != 0) return;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float *row = cm + (qi0 + r) * LD;
            const float m1 = row[DK], l1 = row[DK + 1], m = fmaxf(m_run[r], m1);
            const float c0 = m_run[r] == -INFINITY ? 0.f : expf(m_run[r] - m);
            const float c1 = m1 == -INFINITY ? 0.f : expf(m1 - m);
            l_run[r] = __fmaf_rn(l_run[r], c0, __fmul_rn(l1, c1));
#pragma unroll
            for (int c4 = 0; c4 < OC / 4; ++c4) {
                const float4 p = *reinterpret_cast<const float4 *>(row + 4 * (oc4 + 8 * c4));
                o[r][4 * c4] = __fmaf_rn(o[r][4 * c4], c0, __fmul_rn(p.x, c1));
                o[r][4 * c4 + 1] = __fmaf_rn(o[r][4 * c4 + 1], c0, __fmul_rn(p.y, c1));
                o[r][4 * c4 + 2] = __fmaf_rn(o[r][4 * c4 + 2], c0, __fmul_rn(p.z, c1));
                o[r][4 * c4 + 3] = __fmaf_rn(o[r][4 * c4 + 3], c0, __fmul_rn(p.w, c1));
            }
        }
    }
    // normalize and store the context rows
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int i = i0 + qi0 + r;
        if (i >= T) continue;
        float *dst = a.ctx + ((long long)b * T + i) * (long long)H * DK + (long long)h * DK;
        const float l = l_run[r] > 0.f ? l_run[r] : 1.f;   // a clip of no live frames attends to nothing: zeros
#pragma unroll
        for (int c4 = 0; c4 < OC / 4; ++c4)
            *reinterpret_cast<float4 *>(dst + 4 * (oc4 + 8 * c4)) =
                make_float4(__fdiv_rn(o[r][4 * c4], l), __fdiv_rn(o[r][4 * c4 + 1], l),
                            __fdiv_rn(o[r][4 * c4 + 2], l), __fdiv_rn(o[r][4 * c4 + 3], l));
    }
    grid_launch_dependents();
}

}  // namespace kea
