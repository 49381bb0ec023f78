// kea_lowbit.cu - host side of libkea_lowbit.so: argument checks, the M-bucketed split-K dispatch table,
// TMA descriptor encoding and the launches. The C ABI is declared in include/kea_lowbit.h.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "kea_lowbit.h"
#include "gemm_kernel.cuh"
#include "aux_kernels.cuh"

namespace {

using kea::GemmArgs;

constexpr int kSmsB200 = 148;
constexpr int kMaxDevices = 64;
constexpr int kSmemPerSm = 233472;       // 228 KB of shared memory per SM
constexpr int kMaxDynSmem = 227 * 1024 - 8192;  // leave room for the kernel's static shared memory (< 8 KB)
constexpr int kMaxPortableCluster = 8;
constexpr int kMaxCluster = 16;

int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }
int round_up(int a, int b) { return ceil_div(a, b) * b; }

struct DeviceState {
    bool ready = false;
    int status = KEA_OK;
    int sms = kSmsB200;
};
DeviceState g_devices[kMaxDevices];
std::mutex g_mutex;

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

// One-time per-device set-up: capability check and kernel attributes (not stream work, so it is legal
// inside a CUDA-graph capture; nothing here allocates).
int device_setup(int *device_out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return KEA_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return KEA_ERR_UNSUPPORTED;
    *device_out = dev;
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceState &st = g_devices[dev];
    if (st.ready) return st.status;
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return KEA_ERR_CUDA;
    int status = KEA_OK;
    if (major != 10 || minor != 0) status = KEA_ERR_NO_DEVICE;
    if (status == KEA_OK && !g_encode) {
        cudaDriverEntryPointQueryResult q;
        void *fn = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            status = KEA_ERR_CUDA;
        else
            g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
    if (status == KEA_OK) {
        const void *kernels[6] = {(const void *)kea::lowbit_gemm_kernel<1, 1>, (const void *)kea::lowbit_gemm_kernel<1, 2>,
                                  (const void *)kea::lowbit_gemm_kernel<1, 3>, (const void *)kea::lowbit_gemm_kernel<2, 1>,
                                  (const void *)kea::lowbit_gemm_kernel<2, 2>, (const void *)kea::lowbit_gemm_kernel<2, 3>};
        for (const void *k : kernels) {
            if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem) != cudaSuccess ||
                cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
                status = KEA_ERR_CUDA;
        }
        if (cudaFuncSetAttribute((const void *)kea::quantize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 64 * 1024) != cudaSuccess)
            status = KEA_ERR_CUDA;
    }
    st.status = status;
    st.sms = sms > 0 ? sms : kSmsB200;
    st.ready = true;
    return status;
}

// ---- configuration ---------------------------------------------------------------------------------------
int stage_bytes(int tile_m, int tile_n, int parts, int wbits) {
    const int act = (tile_m / kea::kBM) * parts * kea::kActTileBytes;
    return round_up(act + tile_n * kea::kBK + (tile_n / kea::kPanelN) * wbits * kea::kPanelSubBytes, 1024);
}

uint32_t tmem_columns(int tile_m, int tile_n, int parts) {
    uint32_t need = (uint32_t)((tile_m / kea::kBM) * parts * tile_n), cols = 32;
    while (cols < need) cols <<= 1;
    return cols;
}

int exchange_bytes(int tile_m, int tile_n, int parts) { return (tile_m / kea::kBM) * parts * tile_n * kea::kBM * 4; }

int dyn_smem_bytes(int tile_m, int tile_n, int parts, int wbits, int splits, int stages) {
    int bytes = stages * stage_bytes(tile_m, tile_n, parts, wbits);
    if (splits > 1) bytes = std::max(bytes, exchange_bytes(tile_m, tile_n, parts));
    bytes += 1024;  // alignment slack for the 1024-byte swizzle atoms
    // Never let more CTAs share an SM than its 512 TMEM columns can serve: a CTA waiting in tcgen05.alloc
    // while its cluster peers wait for it could otherwise deadlock.
    const uint32_t cols = tmem_columns(tile_m, tile_n, parts);
    const int max_ctas = std::max(1, (int)(512 / cols));
    const int floor_bytes = kSmemPerSm / (max_ctas + 1) + 1;
    return std::max(bytes, floor_bytes);
}

int max_stages(int tile_m, int tile_n, int parts, int wbits) {
    int s = kea::kMaxStages;
    while (s > 1 && s * stage_bytes(tile_m, tile_n, parts, wbits) + 1024 > kMaxDynSmem) --s;
    return s;
}

// The M-bucketed split-K dispatch table.
//  * M <= 128: one 128-token tile; 128 channels per CTA; K split over a cluster so the grid covers the SMs.
//  * M <= 256 (and P = 1): 256 tokens per CTA, so the weights of a 128-channel tile are expanded once for both halves.
//  * larger M: 256-token x 128-channel tiles, split only when the tile grid is too small to fill the GPU.
KeaGemmConfig choose(int m, int n, int k, int wbits, int parts, int sms) {
    KeaGemmConfig c{};
    const int kb = ceil_div(k, kea::kBK), nt = ceil_div(n, kea::kPanelN);
    const int tile_n = 128;
    const int tile_m = (m > 128 && parts == 1) ? 256 : 128;
    const int tiles = ceil_div(std::max(m, 1), tile_m) * nt;
    int splits = 1;
    if (tiles < sms) splits = std::max(1, sms / tiles);
    splits = std::min({splits, kb, kMaxPortableCluster});
    while (splits > 1 && exchange_bytes(tile_m, tile_n, parts) + 1024 > kMaxDynSmem) --splits;
    const int per = ceil_div(kb, splits);
    int stages = std::min({per, 4, max_stages(tile_m, tile_n, parts, wbits)});
    c.tile_m = tile_m;
    c.tile_n = tile_n;
    c.splits = splits;
    c.stages = std::max(stages, 1);
    c.smem_bytes = dyn_smem_bytes(tile_m, tile_n, parts, wbits, splits, c.stages);
    return c;
}

int check_config(const KeaGemmConfig &c, int n, int k, int parts, int wbits) {
    const int kb = ceil_div(k, kea::kBK), nt = ceil_div(n, kea::kPanelN);
    if (c.tile_m != 128 && c.tile_m != 256) return KEA_ERR_UNSUPPORTED;
    if (c.tile_n != 128 && c.tile_n != 256) return KEA_ERR_UNSUPPORTED;
    if (c.tile_n == 256 && nt % 2) return KEA_ERR_UNSUPPORTED;   // the second panel tile must exist
    if ((c.tile_m / kea::kBM) * parts * c.tile_n > 512) return KEA_ERR_UNSUPPORTED;   // TMEM columns
    if (c.splits < 1 || c.splits > kMaxCluster || c.splits > kb) return KEA_ERR_UNSUPPORTED;
    if (c.stages < 1 || c.stages > kea::kMaxStages) return KEA_ERR_UNSUPPORTED;
    if (c.smem_bytes > kMaxDynSmem) return KEA_ERR_UNSUPPORTED;
    (void)wbits;
    return KEA_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" {

int kea_lowbit_version(void) { return KEA_LOWBIT_VERSION; }

const char *kea_lowbit_status_string(int status) {
    switch (status) {
        case KEA_OK: return "success";
        case KEA_ERR_INVALID_VALUE: return "invalid argument";
        case KEA_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
        case KEA_ERR_UNSUPPORTED: return "unsupported configuration";
        case KEA_ERR_INVALID_CODES: return "invalid packed codes";
        case KEA_ERR_CUDA: return "CUDA call failed";
        case KEA_ERR_NO_DEVICE: return "current device is not an sm_100 GPU";
        case KEA_ERR_DEVICE_TIMEOUT: return "a kernel wait timed out";
        case KEA_ERR_CAPTURE: return "first use of a device during stream capture";
        default: return "unknown status";
    }
}

size_t kea_lowbit_panel_bytes(int32_t wbits, int32_t n, int32_t k) {
    if ((wbits != 1 && wbits != 2) || n < 1 || k < 1) return 0;
    return (size_t)ceil_div(n, kea::kPanelN) * (size_t)ceil_div(k, kea::kBK) * (size_t)wbits * kea::kPanelSubBytes;
}

int kea_lowbit_choose_config(int32_t m, int32_t n, int32_t k, int32_t wbits, int32_t parts, KeaGemmConfig *out) {
    if (!out || m < 0 || n < 1 || k < 1 || (wbits != 1 && wbits != 2) || parts < 1 || parts > 3) return KEA_ERR_INVALID_VALUE;
    int dev = 0, sms = kSmsB200;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sms = v;
    }
    cudaGetLastError();  // a CPU-only process reports no device here; the table then assumes a B200
    *out = choose(m, n, k, wbits, parts, sms);
    return KEA_OK;
}

int kea_lowbit_prepare(const uint8_t *codes, int32_t wbits, int32_t n, int32_t k, uint8_t *panels, uint32_t *error_word,
                       void *stream) {
    if (!codes || !panels || (wbits != 1 && wbits != 2) || n < 1 || k < 1) return KEA_ERR_INVALID_VALUE;
    if (!aligned16(panels)) return KEA_ERR_ALIGNMENT;
    int dev = 0;
    const int st = device_setup(&dev);
    if (st != KEA_OK) return st;
    const int row_bytes = ceil_div((long long)k * wbits, 8);
    const int kb = ceil_div(k, kea::kBK);
    const long long chunks = (long long)ceil_div(n, kea::kPanelN) * kb * wbits * kea::kPanelN;
    const unsigned blocks = (unsigned)((chunks + 255) / 256);
    kea::prepare_panels_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(codes, row_bytes, wbits, n, k, kb, chunks,
                                                                          panels, error_word);
    return cudaGetLastError() == cudaSuccess ? KEA_OK : KEA_ERR_CUDA;
}

int kea_lowbit_quantize(const KeaQuantizeDesc *d, void *stream) {
    if (!d || !d->x || !d->q || !d->qs || d->m < 0 || d->k < 1 || d->parts < 1 || d->parts > 3 || d->t < 1 ||
        d->ldq < d->k)
        return KEA_ERR_INVALID_VALUE;
    if ((long long)d->k * 4 > 64 * 1024) return KEA_ERR_UNSUPPORTED;
    if (d->m == 0) return KEA_OK;
    int dev = 0;
    const int st = device_setup(&dev);
    if (st != KEA_OK) return st;
    kea::QuantArgs a{};
    a.x = d->x;
    a.xb = d->xb;
    a.xt = d->xt;
    a.xk = d->xk;
    a.t = d->t;
    a.M = d->m;
    a.K = d->k;
    a.parts = d->parts;
    a.ldq = d->ldq;
    a.q = d->q;
    a.q_stride = d->q_part_stride;
    a.qs = d->qs;
    a.qs_stride = d->qs_part_stride;
    a.nw = d->norm_weight;
    a.nb = d->norm_bias;
    a.eps = d->eps;
    a.flags = d->flags;
    kea::quantize_kernel<<<d->m, kea::kQuantThreads, d->k * sizeof(float), (cudaStream_t)stream>>>(a);
    return cudaGetLastError() == cudaSuccess ? KEA_OK : KEA_ERR_CUDA;
}

int kea_lowbit_gemm(const KeaGemmDesc *d, void *stream) {
    if (!d) return KEA_ERR_INVALID_VALUE;
    if (d->m < 0 || d->n < 1 || d->k < 1 || d->parts < 1 || d->parts > 3 || (d->wbits != 1 && d->wbits != 2) ||
        (d->y_dtype != KEA_OUT_F32 && d->y_dtype != KEA_OUT_F16))
        return KEA_ERR_INVALID_VALUE;
    if (d->m == 0) return KEA_OK;
    if (!d->q || !d->qs || !d->panels || !d->alpha || !d->y || d->ldy < d->n || d->ldq < d->k) return KEA_ERR_INVALID_VALUE;
    if (d->acc && (d->ld_acc < d->n || (d->parts > 1 && d->acc_part_stride < (int64_t)d->m * d->ld_acc)))
        return KEA_ERR_INVALID_VALUE;
    if (!aligned16(d->q) || d->ldq % 16 || !aligned16(d->panels)) return KEA_ERR_ALIGNMENT;
    if (d->parts > 1 && (d->q_part_stride % 16 || d->q_part_stride < (int64_t)d->m * d->ldq)) return KEA_ERR_ALIGNMENT;
    if (d->flags & ~(KEA_FLAG_SILU | KEA_FLAG_ORDER1 | KEA_FLAG_PDL)) return KEA_ERR_INVALID_VALUE;

    int dev = 0;
    const int st = device_setup(&dev);
    if (st != KEA_OK) return st;

    KeaGemmConfig c = choose(d->m, d->n, d->k, d->wbits, d->parts, g_devices[dev].sms);
    if (d->tile_m || d->tile_n || d->splits || d->stages) {
        if (d->tile_m) c.tile_m = d->tile_m;
        if (d->tile_n) c.tile_n = d->tile_n;
        if (d->splits) c.splits = d->splits;
        if (d->stages) {
            c.stages = d->stages;
        } else {
            const int per = ceil_div(ceil_div(d->k, kea::kBK), std::max(1, c.splits));
            c.stages = std::max(1, std::min({per, 4, max_stages(c.tile_m, c.tile_n, d->parts, d->wbits)}));
        }
        c.smem_bytes = dyn_smem_bytes(c.tile_m, c.tile_n, d->parts, d->wbits, c.splits, c.stages);
    }
    const int cs = check_config(c, d->n, d->k, d->parts, d->wbits);
    if (cs != KEA_OK) return cs;

    // Activations: a 3-D tensor (k, m, part) of int8, tiles of 128 k x 128 rows x 1 part, 128-byte
    // swizzle (the tcgen05 K-major layout). Columns >= k and rows >= m read as zero.
    CUtensorMap qmap;
    const cuuint64_t dims[3] = {(cuuint64_t)d->k, (cuuint64_t)d->m, (cuuint64_t)d->parts};
    const long long pstride = d->parts > 1 ? d->q_part_stride : (long long)d->m * d->ldq;
    const cuuint64_t strides[2] = {(cuuint64_t)d->ldq, (cuuint64_t)std::max<long long>(pstride, 16)};
    const cuuint32_t box[3] = {(cuuint32_t)kea::kBK, (cuuint32_t)kea::kBM, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (g_encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(d->q), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return KEA_ERR_CUDA;

    GemmArgs a{};
    a.panels = d->panels;
    a.qs = d->qs;
    a.qs_stride = d->qs_part_stride;
    a.alpha = d->alpha;
    a.bias = d->bias;
    a.y = d->y;
    a.ldy = d->ldy;
    a.y_f16 = d->y_dtype == KEA_OUT_F16;
    a.acc = d->acc;
    a.ld_acc = d->ld_acc;
    a.acc_stride = d->acc_part_stride;
    a.M = d->m;
    a.N = d->n;
    a.K = d->k;
    a.parts = d->parts;
    a.tile_n = c.tile_n;
    a.tm_blocks = c.tile_m / kea::kBM;
    a.splits = c.splits;
    a.stages = c.stages;
    a.kb_total = ceil_div(d->k, kea::kBK);
    a.flags = d->flags & (KEA_FLAG_SILU | KEA_FLAG_ORDER1);
    a.tmem_cols = tmem_columns(c.tile_m, c.tile_n, d->parts);
    a.stage_bytes = (uint32_t)stage_bytes(c.tile_m, c.tile_n, d->parts, d->wbits);
    const int esize = d->y_dtype == KEA_OUT_F16 ? 2 : 4;
    a.vec_y = aligned16(d->y) && ((d->ldy * esize) % 16 == 0);
    a.vec_acc = d->acc && aligned16(d->acc) && ((d->ld_acc * 4) % 16 == 0) && ((d->acc_part_stride * 4) % 16 == 0);
    a.err = d->error_word;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(d->n, c.tile_n), (unsigned)ceil_div(d->m, c.tile_m), (unsigned)c.splits);
    cfg.blockDim = dim3(kea::kThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)c.smem_bytes;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attrs[2];
    unsigned na = 0;
    if (c.splits > 1) {
        attrs[na].id = cudaLaunchAttributeClusterDimension;
        attrs[na].val.clusterDim.x = 1;
        attrs[na].val.clusterDim.y = 1;
        attrs[na].val.clusterDim.z = (unsigned)c.splits;
        ++na;
    }
    if (d->flags & KEA_FLAG_PDL) {
        attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    cudaError_t e;
    switch (d->wbits * 4 + d->parts) {
        case 5: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<1, 1>, qmap, a); break;
        case 6: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<1, 2>, qmap, a); break;
        case 7: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<1, 3>, qmap, a); break;
        case 9: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<2, 1>, qmap, a); break;
        case 10: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<2, 2>, qmap, a); break;
        default: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<2, 3>, qmap, a); break;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return KEA_ERR_CUDA;
    }
    return KEA_OK;
}

int kea_lowbit_read_error(uint32_t *out) {
    if (!out) return KEA_ERR_INVALID_VALUE;
    int dev = 0;
    const int st = device_setup(&dev);
    if (st != KEA_OK) return st;
    uint32_t v = 0;
    if (cudaMemcpyFromSymbol(&v, kea::g_device_error, sizeof(v)) != cudaSuccess) return KEA_ERR_CUDA;
    const uint32_t zero = 0;
    if (cudaMemcpyToSymbol(kea::g_device_error, &zero, sizeof(zero)) != cudaSuccess) return KEA_ERR_CUDA;
    *out = v;
    return KEA_OK;
}

}  // extern "C"
