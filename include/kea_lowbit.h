/*
 * kea_lowbit.h - C ABI of the B200 (sm_100a) low-bit GEMM library `libkea_lowbit.so`.
 *
 * The library multiplies INT8 activation parts by 1-bit (sign) or 2-bit (ternary) packed weights on the
 * tcgen05 tensor cores (kind::i8, INT32 accumulators in tensor memory) and applies the kea-kernels FP32
 * epilogue. Every entry point takes plain device pointers, sizes and a CUDA stream passed as `void *`
 * (a `cudaStream_t`; NULL is the legacy default stream). Nothing here allocates device memory or
 * synchronizes the host, except `kea_lowbit_read_error`, which says so.
 *
 * Reference interfaces replaced (paths inside the kea-kernels project):
 *   - the NVRTC launch path `_nvrtc.load(...).launch(...)` (src/kea_kernels/_nvrtc.py:116-137), which the
 *     Python layer called with 16 typed kernel arguments (src/kea_kernels/binary/layer.py:196-201);
 *   - the Triton launches of `_quantize` / `_int8_dot` / `_finish` (src/kea_kernels/ternary/fused_kernels.py:
 *     139-160; src/kea_kernels/ternary/encoder4.py:120-148).
 * All status codes are `int`; 0 is success.
 */
#ifndef KEA_LOWBIT_H
#define KEA_LOWBIT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KEA_LOWBIT_VERSION 5

/* Status codes. The Python layer maps 1-4 to ValueError and 5-8 to RuntimeError, as the reference raises
 * ValueError for argument errors (src/kea_kernels/binary/layer.py:66-78,188-189) and RuntimeError for a failed
 * launch (src/kea_kernels/_nvrtc.py:123-124). */
enum {
    KEA_OK = 0,
    KEA_ERR_INVALID_VALUE = 1,   /* a NULL pointer, a non-positive size, an unknown enum value */
    KEA_ERR_ALIGNMENT = 2,       /* a pointer or stride that is not 16-byte aligned where TMA needs it */
    KEA_ERR_UNSUPPORTED = 3,     /* a valid request outside what the kernels implement (e.g. parts = 4) */
    KEA_ERR_INVALID_CODES = 4,   /* prepare: nonzero tail bits, or the unused ternary pattern 0b11 */
    KEA_ERR_CUDA = 5,            /* a CUDA runtime / driver call failed (launch, attribute, tensor map) */
    KEA_ERR_NO_DEVICE = 6,       /* the current device is not an sm_100 (B200-class) GPU */
    KEA_ERR_DEVICE_TIMEOUT = 7,  /* a kernel's bounded wait expired and the kernel returned early */
    KEA_ERR_CAPTURE = 8,         /* first use of a device inside a CUDA-graph capture (one-time set-up needed) */
    KEA_ERR_SCRATCH_LIMIT = 9    /* kea_lowbit_gemm_noalloc: the shape's split-K scratch exceeds its static buffer */
};

/* Output element type of y. FP32 is the reference's output (src/kea_kernels/binary/kernels.py:315-325);
 * FP16 is round-to-nearest-even of the same FP32 value. */
enum { KEA_OUT_F32 = 0, KEA_OUT_F16 = 1 };

/* kea_lowbit_gemm flags. SILU and ORDER1 are the reference's `flags` bits 0 and 1
 * (src/kea_kernels/binary/kernels.py:73-84: bit 0 SiLU epilogue, bit 1 the other P = 2 contraction order). */
enum {
    KEA_FLAG_SILU = 1,
    KEA_FLAG_ORDER1 = 2,
    KEA_FLAG_PDL = 4,           /* launch with programmatic dependent launch (overlap with the previous kernel) */
    KEA_FLAG_NO_PAIR = 8,       /* never use the persistent CTA-pair kernel (the per-tile kernel runs instead) */
    KEA_FLAG_FORCE_PAIR = 16,   /* the pair kernel wherever its shape allows (1-2 parts, N % 256 == 0, m > 256,
                                   k <= 32768), also where the table would take the per-tile kernel */
    KEA_FLAG_FORCE_SWAP = 32,   /* the small-M swapped-operand kernel (weights on the MMA's M axis, tokens on N) at any
                                   shape; `tile_m` (its token tile: a multiple of 16 up to 256 / parts), `splits` and
                                   `stages` (0: the table's) then apply to it; tile_n must be 0 */
    KEA_FLAG_NO_SWAP = 64,      /* keep the table off the swapped-operand kernel (128-token tiles run instead) */
    KEA_FLAG_TEST_STALL = 128,  /* tests only, with KEA_FLAG_FORCE_SWAP: the kernel's producer issues no activation
                                   copy, so its MMA warp's bounded wait runs out (see wait_clocks), the kernel reports
                                   KEA_DEVERR_TIMEOUT and returns; the output is left undefined */
    KEA_FLAG_NO_RESIDENT_WEIGHTS = 256,  /* the pair kernel re-expands the weights of every tile it visits, also where
                                            (one part, K <= 1024) it would keep a channel tile's weights resident */
    KEA_FLAG_FORCE_REG = 512,   /* the small-M register-operand kernel (warp-level MMAs, weights expanded in registers) at
                                   any shape; `tile_n` (channels per CTA: 16, 32, 64 or 128), `tile_m` (activation rows
                                   per CTA, tokens x parts: 16 or 32) and `splits` (K-slices among its 8 warps: 1, 2, 4
                                   or 8) then apply to it (0: the table's); stages must be 0 */
    KEA_FLAG_NO_REG = 1024      /* keep the table off the register-operand kernel (its tcgen05 choice runs instead) */
};

/* Device error word bits (written by kernels into `error_word`, or into the library's own device word). */
enum {
    KEA_DEVERR_TIMEOUT = 1,      /* an mbarrier wait exceeded its bound */
    KEA_DEVERR_TAIL_BITS = 2,    /* prepare: nonzero padding bits past K */
    KEA_DEVERR_TERNARY_11 = 4    /* prepare: a 2-bit field holds the unused pattern 0b11 */
};

/*
 * One low-bit GEMM:
 *   acc_c[m, n] = sum_k q_c[m, k] * w[n, k]            (exact INT32; w in {-1,+1} or {-1,0,+1})
 *   r           = comb_P(acc, qs)                       (P = parts; see below)
 *   y[m, n]     = bias ? fma(r, alpha[n], bias[n]) : r * alpha[n],   then SiLU if KEA_FLAG_SILU
 * comb_1 = RN(float(acc_0) * s_0); comb_2 = fma(acc_0, s_0, RN(acc_1 * s_1)) (ORDER1: fma(acc_1, s_1,
 * RN(acc_0 * s_0))); comb_3 = fma(acc_2, s_2, comb_2). Every operation is one IEEE FP32 rounding, as in
 * the reference's comb<P> / epilogue_p (src/kea_kernels/binary/kernels_parts.py:30-45).
 *
 * Replaces Int8MmaLayer.dot / dot_parts -> b1_dot (src/kea_kernels/binary/layer.py:182-209;
 * src/kea_kernels/binary/layer_parts.py:112-130; src/kea_kernels/binary/kernels.py:556-564) and the ternary
 * _int8_dot + _finish launches (src/kea_kernels/ternary/fused_kernels.py:53-120,139-160).
 */
typedef struct KeaGemmDesc {
    const int8_t *q;          /* int8 [parts][m][ldq]; k columns are read, columns >= k are ignored */
    int64_t q_part_stride;    /* elements between parts (multiple of 16 when parts > 1) */
    int32_t ldq;              /* row stride in elements, multiple of 16 (q must be 16-byte aligned) */
    int32_t parts;            /* 1, 2 or 3 residual INT8 parts */
    const float *qs;          /* FP32 [parts][m] per-token part scales */
    int64_t qs_part_stride;   /* elements between parts of qs */
    const uint8_t *panels;    /* weights prepared by kea_lowbit_prepare */
    int32_t wbits;            /* 1 (signs) or 2 (ternary) */
    int32_t n, k;             /* output channels, reduction length */
    const float *alpha;       /* FP32 [n] per-channel weight scale */
    const float *bias;        /* FP32 [n] or NULL */
    void *y;                  /* [m][ldy] FP32 or FP16 */
    int64_t ldy;              /* row stride of y in elements */
    int32_t y_dtype;          /* KEA_OUT_F32 or KEA_OUT_F16 */
    int32_t *acc;             /* optional INT32 [parts][m][ld_acc] accumulators, or NULL */
    int64_t ld_acc;           /* row stride of acc in elements */
    int64_t acc_part_stride;  /* elements between parts of acc */
    int32_t m;                /* tokens (rows of q and y); 0 is a no-op */
    int32_t flags;            /* KEA_FLAG_* */
    int32_t tile_m;           /* 0: dispatch table; 128 or 256: tokens per CTA of the per-tile tcgen05 kernel (any
                                 forced field selects it); 1..16: the CUDA-core kernel (m <= 16, splits and stages
                                 0 or 1) */
    int32_t tile_n;           /* 0: dispatch table; else channels per CTA (32, 64, 128 or 256; 8, 16 or 32 for the
                                 CUDA-core kernel) */
    int32_t splits;           /* 0: dispatch table; else split-K ways = cluster size (1..16) */
    int32_t stages;           /* 0: dispatch table; else pipeline stages (1..8) */
    uint32_t *error_word;     /* device word OR-ed with KEA_DEVERR_* bits, or NULL for the library's own */
    const float *residual;    /* NULL, or FP32 [m][ld_residual]: y = residual + residual_scale * (the epilogue's
                                 value), two IEEE roundings as `residual + scale * y` in PyTorch; FP32 y only. May be
                                 y itself: every element is read before it is written, by the same thread */
    int64_t ld_residual;
    float residual_scale;
    void *workspace;          /* NULL, or device scratch of workspace_bytes (16-byte aligned) for split-K of the pair
                                 kernel: where a shape has too few 256 x 256 tiles to occupy the GPU, its K range is
                                 cut into slices whose INT32 partial sums go here and are finished by a second kernel
                                 (same bits). kea_lowbit_workspace_bytes says how much a shape uses; with less (or
                                 NULL) the GEMM runs unsplit. Calls sharing a workspace must not overlap on the GPU. */
    int64_t workspace_bytes;
    int64_t wait_clocks;      /* 0: the library's bound on a kernel's wait (4e9 SM clocks, about 2 s); else the SM
                                 clocks one wait of the swapped-operand kernel may last before it gives up, reports
                                 KEA_DEVERR_TIMEOUT in the error word and returns (the context stays usable) */
} KeaGemmDesc;

/* Tile configuration picked for a shape (the M-bucketed split-K dispatch table). */
typedef struct KeaGemmConfig {
    int32_t tile_m;           /* tokens per CTA: 128 or 256 (one or two tcgen05 M = 128 blocks) */
    int32_t tile_n;           /* channels per CTA: 32, 64, 128 or 256 (the tcgen05 N dimension) */
    int32_t splits;           /* K split across a thread-block cluster of this size */
    int32_t stages;           /* smem pipeline depth (k128 blocks in flight) */
    int32_t smem_bytes;       /* dynamic shared memory per CTA */
    int32_t kernel;           /* 0: the per-tile tcgen05 kernel; 1: the persistent CTA-pair kernel (tcgen05
                                 cta_group::2, 256 x 256 tiles per pair of SMs, double-buffered accumulators); 2: the
                                 CUDA-core kernel for M <= 16 (tile_n = channels per CTA); 3: the small-M swapped-operand
                                 kernel (tile_m = tokens per token tile, tile_n = 128 channels, splits = cluster along K);
                                 4: the small-M register-operand kernel (tile_m = activation rows per CTA, tile_n =
                                 channels per CTA, splits = K-slices among its warps) */
} KeaGemmConfig;

int kea_lowbit_gemm(const KeaGemmDesc *desc, void *stream);

/* kea_lowbit_gemm for callers that cannot allocate device memory. No counterpart in the reference (whose launcher
 * allocates a workspace with every call). A speech service answering requests in real time may not call cudaMalloc
 * on its request path: cudaMalloc can wait for the whole device and its latency has no bound; and a host that runs
 * this library inside its own memory budget must not have device memory grow behind its back. This entry point
 * allocates nothing: where the dispatch table splits K (few pair tiles, long K), the INT32 partial sums go to a
 * scratch buffer of KEA_NOALLOC_SCRATCH_BYTES (16 MiB) that the library holds in a static device array, present on
 * every GPU that loads the library until the process exits; desc->workspace / workspace_bytes are ignored.
 * The caller still passes every input and output. A shape whose split would need more scratch is refused with
 * KEA_ERR_SCRATCH_LIMIT (kea_lowbit_workspace_bytes says how much a shape needs); shapes that do not split need none.
 * The buffer's device address is looked up in the one-time set-up of each device, which the first call of any entry
 * point on that device runs (this one included): make that first call before any stream capture (inside one it
 * returns KEA_ERR_CAPTURE). All calls on a device share its one buffer, which keeps the last call's contents (nothing in it needs
 * to start at zero: each call writes every partial sum it later reads), so calls on that device that overlap on the
 * GPU (for example on two streams) race: keep them on one stream or order them with events. */
#define KEA_NOALLOC_SCRATCH_BYTES (16u << 20)
int kea_lowbit_gemm_noalloc(const KeaGemmDesc *desc, void *stream);

/* The configuration kea_lowbit_gemm uses when tile_m / tile_n / splits / stages are 0.
 * Replaces configs.choose (src/kea_kernels/binary/configs.py:53-58). */
int kea_lowbit_choose_config(int32_t m, int32_t n, int32_t k, int32_t wbits, int32_t parts, KeaGemmConfig *out);

/* Bytes of the prepared panel layout: ceil(n/128) * ceil(k/128) * wbits * 2048.
 * Replaces kernels.fragment_bytes (src/kea_kernels/binary/kernels.py:726-727). */
size_t kea_lowbit_panel_bytes(int32_t wbits, int32_t n, int32_t k);

/* Scratch bytes kea_lowbit_gemm uses for split-K at this shape under the dispatch table (0: none):
 * slices x parts x m x n x 4. Replaces the reference's per-call workspace sizing
 * (src/kea_kernels/binary/kernels.py:640-700, DotConfig workspace; allocated per call at layer.py:194-195). */
size_t kea_lowbit_workspace_bytes(int32_t m, int32_t n, int32_t k, int32_t wbits, int32_t parts);

/* Re-lays export codes (uint8 [n][ceil(k*wbits/8)] on the device; parakeet-binary-v1 LSB-first signs or
 * parakeet-ternary-v1 2-bit fields) into panels of kea_lowbit_panel_bytes bytes, and checks the codes:
 * nonzero tail bits or a 0b11 field set KEA_DEVERR_* bits in error_word (NULL: the library's own word).
 * Replaces relayout(unpack_bits(codes)) in Int8MmaLayer.prepare (src/kea_kernels/binary/kernels.py:730-742;
 * src/kea_kernels/binary/layer.py:37-56) and PackedLinear's word re-layout (src/kea_kernels/ternary/runtime.py:
 * 33-35). */
int kea_lowbit_prepare(const uint8_t *codes, int32_t wbits, int32_t n, int32_t k, uint8_t *panels,
                       uint32_t *error_word, void *stream);

/* Residual INT8 quantizer:
 *   x[m, kk] at x + (m / t) * xb + (m % t) * xt + kk * xk (elements);
 *   optional LayerNorm over k (norm_weight / norm_bias FP32 [k]), optional input SiLU;
 *   for each part c: s_c = max(amax / 127, 1e-30), q = rint(x / s_c), x -= q * s_c.
 * Division is IEEE round-to-nearest (the CPU oracle reproduces it bit for bit).
 * Replaces b1_quantize (src/kea_kernels/binary/kernels.py:567-617; layer.py:154-165) and the Triton
 * _quantize (src/kea_kernels/ternary/fused_kernels.py:31-50). */
typedef struct KeaQuantizeDesc {
    const float *x;
    int64_t xb, xt, xk;       /* strides in elements (see above) */
    int32_t t;                /* rows per batch entry (>= 1) */
    int32_t m, k, parts;
    int8_t *q;                /* int8 [parts][m][ldq], columns k..ldq-1 written as 0; 4-byte aligned, ldq and the
                                 part stride multiples of 4 (else KEA_ERR_ALIGNMENT) */
    int64_t q_part_stride;
    int32_t ldq;
    float *qs;                /* FP32 [parts][m] */
    int64_t qs_part_stride;
    const float *norm_weight; /* NULL: no LayerNorm */
    const float *norm_bias;
    float eps;
    int32_t flags;            /* KEA_QUANT_* */
    /* Optional LayerNorm applied before everything else - a layer's output norm, as the reference's row epilogue
     * applies OUT_NORM before the next projection's quantizer (src/kea_kernels/ternary/row_fusion.py:27-52) - with
     * its FP32 result written to normed[m][ld_normed] (the next skip connection's input). Needs unit-stride,
     * 16-byte aligned rows (x, normed, both norms' parameters); normed may be x itself (in place). NULL: none. */
    const float *pre_norm_weight;
    const float *pre_norm_bias;  /* NULL: no bias */
    float pre_eps;
    float *normed;
    int64_t ld_normed;        /* elements, a multiple of 4 */
} KeaQuantizeDesc;

enum {
    KEA_QUANT_INPUT_SILU = 1,
    KEA_QUANT_PDL = 2,            /* launch with programmatic dependent launch (overlap with the previous kernel) */
    KEA_QUANT_NARROW_ROWS = 4     /* as few threads per row as registers allow (one warp for K <= 1024): the
                                     reduction order of the GEMM's fused prologue quantizer (kea_lowbit_project) */
};

int kea_lowbit_quantize(const KeaQuantizeDesc *desc, void *stream);

/* Quantize + GEMM in one call: the reference's Int8MmaLayer.project (src/kea_kernels/binary/layer.py:118-151;
 * src/kea_kernels/binary/layer_parts.py:65-90), x -> residual INT8 parts -> the low-bit GEMM with its epilogue.
 * `quant` gives the input rows and the quantizer's options (pre-norm, LayerNorm, input SiLU); its m, k, parts, q, ldq,
 * qs (and the part strides when parts > 1) must equal `gemm`'s, whose q / qs receive the parts. By default the two
 * kernels run back to back (kea_lowbit_quantize with quant's flags, then kea_lowbit_gemm): measured the faster form
 * on B200, since the GEMM's set-up and weight expansion overlap the quantizer kernel under programmatic dependent
 * launch. With KEA_PROJECT_FUSE, where the shape allows - one part, 33 <= m <= 128 (the per-tile route), k a multiple
 * of 128 up to 1024, channel tiles in whole clusters of 8, unit-stride 16-byte-aligned rows, a pre-norm output apart
 * from x - the quantizer runs inside the GEMM kernel, one launch: each cluster of 8 CTAs quantizes the token rows
 * (one warp a row, the arithmetic of kea_lowbit_quantize with KEA_QUANT_NARROW_ROWS, bit for bit) into `scratch`,
 * then reads them back as its activation boxes. scratch: 16-byte aligned, kea_lowbit_project_scratch_bytes(...)
 * bytes (0 = the fused form never applies; a smaller scratch falls back to the two kernels). */
typedef struct KeaProjectDesc {
    KeaGemmDesc gemm;
    KeaQuantizeDesc quant;
    void *scratch;
    size_t scratch_bytes;
    int32_t flags;            /* KEA_PROJECT_* */
} KeaProjectDesc;

enum { KEA_PROJECT_FUSE = 1 };

int kea_lowbit_project(const KeaProjectDesc *desc, void *stream);
/* Which form kea_lowbit_project takes for this descriptor (with its flags): 1 one fused kernel, 0 the two kernels,
 * -(status) when the arguments are refused. Launches nothing. */
int kea_lowbit_project_fuses(const KeaProjectDesc *desc);
size_t kea_lowbit_project_scratch_bytes(int32_t m, int32_t n, int32_t k, int32_t wbits, int32_t parts);

/* The convolution module's middle between its pointwise GEMMs, in one pass over pw1's output:
 *   g[b, t, c] = h[b, t, c] * sigmoid(h[b, t, C + c]), zero where t >= lengths[b] (padding);
 *   y[b, t, c] = bias[c] + sum_j w[c, j] * g[b, t + j - kw / 2, c]   (zero padding in time),
 * h FP32 [B][T][2C] and y FP32 [B][T][C] contiguous, w FP32 [C][kw] (BatchNorm folded in), kw odd <= 31.
 * No reference C counterpart: replaces the reference's Triton glu_pad + torch depthwise conv + batch norm
 * (src/kea_kernels/ternary/layer_fusions4.py:52-77). */
typedef struct KeaConvDesc {
    const float *h;
    float *y;
    const float *weight;      /* [C][kw] */
    const float *bias;        /* [C] or NULL */
    const int32_t *lengths;   /* [B] frames per clip, or NULL */
    int32_t b, t, c, kw;
    int32_t flags;            /* KEA_CONV_* */
    /* Optional: the next projection's quantizer fused in (pw2's: residual INT8 parts of y, or of SiLU(y) with
     * KEA_CONV_QUANT_SILU, with kea_lowbit_quantize's arithmetic, bit for bit): q int8 [parts][b * t][ldq] (columns
     * c .. ldq - 1 written as 0; 4-byte aligned, ldq and the part stride multiples of 4), qs FP32 [parts][b * t].
     * Needs c % 4 == 0, c <= 1024 and 16-byte aligned h. y may then be NULL (not written). q NULL: no quantizer. */
    int8_t *q;
    int64_t q_part_stride;
    int32_t ldq;
    float *qs;
    int64_t qs_part_stride;
    int32_t parts;
} KeaConvDesc;

enum {
    KEA_CONV_PDL = 1,
    KEA_CONV_QUANT_SILU = 2       /* SiLU before the fused quantizer (the conv module's activation) */
};

int kea_lowbit_glu_depthwise(const KeaConvDesc *desc, void *stream);

/* Relative-position self-attention of the FastConformer, FP32, one kernel (online softmax, no T x T buffer):
 *   score[i, j] = ((q_i + bias_u) . k_j + (q_i + bias_v) . pos[j + t - 1 - i]) * scale, keys j >= lengths[b] masked,
 *   ctx_i = softmax_j(score[i, :]) . v_j,
 * qkv FP32 [b][t][3][h][dk] (q, k, v of one token row), pos FP32 [2t - 1][h][dk] (the position projection of the
 * relative positions t - 1 .. -(t - 1)), bias_u / bias_v FP32 [h][dk], ctx FP32 [b][t][h][dk]; dk 32, 64 or 128;
 * 16-byte aligned buffers. No reference C counterpart: replaces the reference's fused relative attention
 * (src/kea_kernels/ternary/fused_kernels.py, relative_attention) and NeMo's RelPositionMultiHeadAttention math. */
typedef struct KeaAttentionDesc {
    const float *qkv;
    const float *pos;
    const float *bias_u, *bias_v;
    const int32_t *lengths;   /* [b] key frames per clip, or NULL */
    float *ctx;
    int32_t b, t, h, dk;
    float scale;
    int32_t flags;            /* KEA_CONV_PDL */
} KeaAttentionDesc;

int kea_lowbit_rel_attention(const KeaAttentionDesc *desc, void *stream);

/* Reads and clears the library's own device error word on the current device. Synchronizes the device. */
int kea_lowbit_read_error(uint32_t *out);

const char *kea_lowbit_status_string(int status);
int kea_lowbit_version(void);

#ifdef __cplusplus
}
#endif

#endif /* KEA_LOWBIT_H */
