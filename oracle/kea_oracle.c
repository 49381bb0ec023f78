/*
 * ORACLE - TEST INFRASTRUCTURE ONLY. Imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg;
 * never by the product (kea-kernels_b200/). It restates on the CPU, in plain C, the arithmetic of kea-kernels'
 * low-bit GEMM path so the CUDA library can be checked against it bit for bit:
 *
 *   - unpack: parakeet-binary-v1 signs (src/kea_kernels/binary/bits.py:41-53: code k = bit k % 8 of byte k // 8,
 *     1 = +1, 0 = -1) and parakeet-ternary-v1 fields (src/kea_kernels/formats.py:73-81: 01 = +1, 10 = -1, 00 = 0,
 *     code k at bits 2 (k % 4) of byte k // 4), rejecting nonzero tail bits and the 11 pattern;
 *   - the integer product acc_c[m, n] = sum_k q_c[m, k] w[n, k], exact (the int64 matmul of the reference's GPU test
 *     oracle, tests/test_kernels_gpu.py:23-27; INT32 is exact here because |acc| <= 127 K < 2^31);
 *   - the FP32 epilogue comb<P> / epilogue_p (src/kea_kernels/binary/kernels_parts.py:30-45): one IEEE rounding per
 *     multiply, fmaf() for each fused multiply-add, bias by fma(r, alpha, bias), then optionally
 *     SiLU y / (1 + exp(-y)) evaluated in double (the GPU's ex2.approx / div.full are checked to a tolerance);
 *   - the residual INT8 quantizer (src/kea_kernels/ternary/fused_kernels.py:31-50 without LayerNorm / SiLU):
 *     s = max(amax / 127, 1e-30), q = rint(x / s), x -= q * s, every division IEEE;
 *   - the B200 panel layout of the prepared weights (this build's own format, checked byte for byte).
 * Compile with -ffp-contract=off so no multiply-add is fused behind the code's back.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <pthread.h>

/* Returns 0, or 1 for nonzero tail bits, 2 for a ternary 11 field. w: int8 [n][k]. */
int kea_oracle_unpack(const uint8_t *codes, int wbits, int n, int k, int8_t *w) {
    const int row_bytes = (k * wbits + 7) / 8;
    const int per_byte = 8 / wbits;
    int status = 0;
    for (int r = 0; r < n; ++r) {
        const uint8_t *src = codes + (long)r * row_bytes;
        for (int b = 0; b < row_bytes; ++b) {
            const unsigned v = src[b];
            for (int f = 0; f < per_byte; ++f) {
                const int kk = b * per_byte + f;
                const unsigned field = (v >> (f * wbits)) & ((1u << wbits) - 1u);
                if (kk >= k) {
                    if (field) status |= 1;
                    continue;
                }
                int8_t val;
                if (wbits == 1) {
                    val = field ? 1 : -1;
                } else {
                    if (field == 3) status |= 2;
                    val = field == 1 ? 1 : (field == 2 ? -1 : 0);
                }
                w[(long)r * k + kk] = val;
            }
        }
    }
    return status;
}

/* Panels: [ceil(n/128)][ceil(k/128)][wbits][4 words][128 rows][4 bytes]; row r of sub-block s of k-block b of tile
 * t holds the 16 export bytes of channel 128 t + r starting at byte 16 wbits b + 16 s (zero past the row end), read
 * as four little-endian words (bytes 4 j .. 4 j + 3 form word j), stored at (j * 128 + r) * 4 within the sub-block
 * after the codes of each word are interleaved: 1 bit - code i (bit i) moves to bit 4 (i % 8) + i / 8; 2 bits -
 * field i (bits 2 i, 2 i + 1) moves to bits 4 (i % 8) + 2 (i / 8), + 1. */
static uint32_t interleave(uint32_t w, int wbits) {
    uint32_t out = 0;
    if (wbits == 1)
        for (int i = 0; i < 32; ++i) out |= ((w >> i) & 1u) << (4 * (i % 8) + i / 8);
    else
        for (int i = 0; i < 16; ++i) out |= ((w >> (2 * i)) & 3u) << (4 * (i % 8) + 2 * (i / 8));
    return out;
}

void kea_oracle_panels(const uint8_t *codes, int wbits, int n, int k, uint8_t *out) {
    const int row_bytes = (k * wbits + 7) / 8;
    const int nt = (n + 127) / 128, kb = (k + 127) / 128;
    long sub = 0;
    for (int t = 0; t < nt; ++t)
        for (int b = 0; b < kb; ++b)
            for (int s = 0; s < wbits; ++s, ++sub)
                for (int r = 0; r < 128; ++r)
                    for (int j = 0; j < 4; ++j) {
                        const int ch = t * 128 + r;
                        uint32_t w = 0;
                        for (int i = 0; i < 4; ++i) {
                            const int byte = b * 16 * wbits + s * 16 + 4 * j + i;
                            if (ch < n && byte < row_bytes) w |= (uint32_t)codes[(long)ch * row_bytes + byte] << (8 * i);
                        }
                        w = interleave(w, wbits);
                        for (int i = 0; i < 4; ++i) out[sub * 2048 + (j * 128 + r) * 4 + i] = (uint8_t)(w >> (8 * i));
                    }
}

static float combine(const int32_t *a, const float *s, int parts, int order) {
    if (parts == 1) return (float)a[0] * s[0];
    float r = order ? fmaf((float)a[1], s[1], (float)a[0] * s[0]) : fmaf((float)a[0], s[0], (float)a[1] * s[1]);
    if (parts == 3) r = fmaf((float)a[2], s[2], r);
    return r;
}

float kea_oracle_finish(const int32_t *a, const float *s, int parts, int flags, float alpha, const float *bias) {
    float r = combine(a, s, parts, (flags >> 1) & 1);
    r = bias ? fmaf(r, alpha, *bias) : r * alpha;
    if (flags & 1) r = (float)((double)r / (1.0 + exp(-(double)r)));
    return r;
}

/* y [m][n] from precomputed accumulators acc [parts][m][n] (the epilogue alone). */
void kea_oracle_finish_all(const int32_t *acc, const float *qs, long qs_stride, int parts, int m, int n,
                           const float *alpha, const float *bias, int flags, float *y) {
    for (int row = 0; row < m; ++row)
        for (int col = 0; col < n; ++col) {
            int32_t a[3] = {0, 0, 0};
            float s[3] = {0.f, 0.f, 0.f};
            for (int p = 0; p < parts; ++p) {
                a[p] = acc[(long)p * m * n + (long)row * n + col];
                s[p] = qs[p * qs_stride + row];
            }
            y[(long)row * n + col] = kea_oracle_finish(a, s, parts, flags, alpha[col], bias ? bias + col : 0);
        }
}

struct gemm_job {
    const int8_t *q;
    long q_stride;
    int ldq, parts;
    const float *qs;
    long qs_stride;
    const int8_t *w;
    int n, k;
    const float *alpha, *bias;
    int m, flags;
    float *y;
    int32_t *acc;
    int row0, row1;
};

static void *gemm_rows(void *arg) {
    const struct gemm_job *j = (const struct gemm_job *)arg;
    for (int row = j->row0; row < j->row1; ++row) {
        for (int col = 0; col < j->n; ++col) {
            int32_t a[3] = {0, 0, 0};
            float s[3] = {0.f, 0.f, 0.f};
            const int8_t *wr = j->w + (long)col * j->k;
            for (int p = 0; p < j->parts; ++p) {
                const int8_t *qr = j->q + p * j->q_stride + (long)row * j->ldq;
                int32_t sum = 0;
                for (int kk = 0; kk < j->k; ++kk) sum += (int32_t)qr[kk] * (int32_t)wr[kk];
                a[p] = sum;
                s[p] = j->qs[p * j->qs_stride + row];
                if (j->acc) j->acc[(long)p * j->m * j->n + (long)row * j->n + col] = sum;
            }
            j->y[(long)row * j->n + col] =
                kea_oracle_finish(a, s, j->parts, j->flags, j->alpha[col], j->bias ? j->bias + col : 0);
        }
    }
    return 0;
}

/* y [m][n] FP32 and (optional) acc [parts][m][n]; q [parts][m][ldq] (part stride q_stride), qs [parts][m]
 * (part stride qs_stride); w int8 [n][k]. Rows are split over `threads` POSIX threads. */
void kea_oracle_gemm(const int8_t *q, long q_stride, int ldq, int parts, const float *qs, long qs_stride,
                     const int8_t *w, int n, int k, const float *alpha, const float *bias, int m, int flags, float *y,
                     int32_t *acc, int threads) {
    enum { kMaxThreads = 256 };
    if (threads < 1) threads = 1;
    if (threads > kMaxThreads) threads = kMaxThreads;
    if (threads > m) threads = m > 0 ? m : 1;
    struct gemm_job jobs[kMaxThreads];
    pthread_t tids[kMaxThreads];
    for (int t = 0; t < threads; ++t) {
        struct gemm_job j = {q, q_stride, ldq, parts, qs, qs_stride, w, n, k, alpha, bias, m, flags, y, acc,
                             (int)((long)m * t / threads), (int)((long)m * (t + 1) / threads)};
        jobs[t] = j;
    }
    int started = 0;
    for (int t = 1; t < threads; ++t) {
        if (pthread_create(&tids[t], 0, gemm_rows, &jobs[t]) != 0) break;
        started = t;
    }
    gemm_rows(&jobs[0]);
    for (int t = 1; t <= started; ++t) pthread_join(tids[t], 0);
    for (int t = started + 1; t < threads; ++t) gemm_rows(&jobs[t]);  /* rows of threads that failed to start */
}

/* x [m][k] FP32 -> q [parts][m][ldq] (zero past k), qs [parts][m]. */
int kea_oracle_quantize(const float *x, int m, int k, int parts, int8_t *q, int ldq, float *qs) {
    float *r = (float *)malloc(sizeof(float) * (size_t)k);
    if (!r) return 1;
    for (int row = 0; row < m; ++row) {
        memcpy(r, x + (long)row * k, sizeof(float) * (size_t)k);
        for (int p = 0; p < parts; ++p) {
            float amax = 0.f;
            for (int kk = 0; kk < k; ++kk) amax = fmaxf(amax, fabsf(r[kk]));
            float scale = amax / 127.0f;
            if (scale < 1.0e-30f) scale = 1.0e-30f;
            int8_t *dst = q + (long)p * m * ldq + (long)row * ldq;
            for (int kk = 0; kk < ldq; ++kk) {
                if (kk < k) {
                    const float v = rintf(r[kk] / scale);
                    dst[kk] = (int8_t)(int)v;
                    r[kk] = r[kk] - v * scale;
                } else {
                    dst[kk] = 0;
                }
            }
            qs[(long)p * m + row] = scale;
        }
    }
    free(r);
    return 0;
}
