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
#include "gemm_pair_kernel.cuh"
#include "gemm_pair_ws_kernel.cuh"
#include "gemm_swap_kernel.cuh"
#include "gemv_kernel.cuh"
#include "gemm_reg_kernel.cuh"
#include "conv_kernels.cuh"
#include "attention_kernels.cuh"
#include "aux_kernels.cuh"

namespace {

using kea::GemmArgs;

constexpr int kSmsB200 = 148;
constexpr int kMaxDevices = 64;
constexpr int kSmemPerSm = 233472;       // 228 KB of shared memory per SM
constexpr int kMaxDynSmem = 227 * 1024 - 8192;  // leave room for the kernel's static shared memory (< 8 KB)
// The pair kernel's static shared memory is a few hundred bytes, so its dynamic share may reach 226 KB.
constexpr int kPairMaxDynSmem = 227 * 1024 - 1024;
constexpr int kMaxPortableCluster = 8;
constexpr int kRegMaxSmem = 64 * 1024;   // the register-operand kernel's partial sums (at most ~37 KB in use)
constexpr int kMaxCluster = 16;

int ceil_div(long long a, long long b) { return (int)((a + b - 1) / b); }
int round_up(int a, int b) { return ceil_div(a, b) * b; }

struct DeviceState {
    bool ready = false;
    int status = KEA_OK;
    int sms = kSmsB200;
    void *noalloc_scratch = nullptr;   // device address of g_noalloc_scratch on this device
};
DeviceState g_devices[kMaxDevices];
std::mutex g_mutex;

// Split-K partial sums for kea_lowbit_gemm_noalloc, in a static device array so that its callers allocate nothing.
// Host code must not use the array's name as a device address (on the host it names a stand-in); the address comes
// from cudaGetSymbolAddress, looked up in the one-time set-up of each device with that device current.
static __device__ __align__(256) int g_noalloc_scratch[KEA_NOALLOC_SCRATCH_BYTES / sizeof(int)];

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;

// One-time per-device set-up: capability check, kernel attributes and the no-allocation scratch address. Nothing here
// allocates, but it loads the library's kernels onto the device, which a stream capture may not see happen: an entry
// point called for the first time on a device while `stream` is capturing returns KEA_ERR_CAPTURE instead.
int device_setup(int *device_out, void *stream, bool check_capture = true) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return KEA_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return KEA_ERR_UNSUPPORTED;
    *device_out = dev;
    std::lock_guard<std::mutex> lock(g_mutex);
    DeviceState &st = g_devices[dev];
    if (st.ready) return st.status;
    if (check_capture) {
        cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing((cudaStream_t)stream, &capturing) != cudaSuccess) {
            cudaGetLastError();
            return KEA_ERR_CUDA;
        }
        if (capturing != cudaStreamCaptureStatusNone) return KEA_ERR_CAPTURE;
    }
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
        const void *pair_kernels[4] = {(const void *)kea::lowbit_gemm_pair_kernel<1, 1>,
                                       (const void *)kea::lowbit_gemm_pair_kernel<2, 1>,
                                       (const void *)kea::lowbit_gemm_pair_kernel<1, 2>,
                                       (const void *)kea::lowbit_gemm_pair_kernel<2, 2>};
        for (const void *k : pair_kernels)
            if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairMaxDynSmem) != cudaSuccess)
                status = KEA_ERR_CUDA;
        const void *ws_kernels[2] = {(const void *)kea::lowbit_gemm_pair_ws_kernel<1>,
                                     (const void *)kea::lowbit_gemm_pair_ws_kernel<2>};
        for (const void *k : ws_kernels)
            if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kPairMaxDynSmem) != cudaSuccess)
                status = KEA_ERR_CUDA;
        const void *swap_kernels[6] = {
            (const void *)kea::lowbit_gemm_swap_kernel<1, 1>, (const void *)kea::lowbit_gemm_swap_kernel<1, 2>,
            (const void *)kea::lowbit_gemm_swap_kernel<1, 3>, (const void *)kea::lowbit_gemm_swap_kernel<2, 1>,
            (const void *)kea::lowbit_gemm_swap_kernel<2, 2>, (const void *)kea::lowbit_gemm_swap_kernel<2, 3>};
        for (const void *k : swap_kernels) {
            if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem) != cudaSuccess ||
                cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
                status = KEA_ERR_CUDA;
        }
        if (cudaFuncSetAttribute((const void *)kea::quantize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 64 * 1024) != cudaSuccess)
            status = KEA_ERR_CUDA;
        const void *attn_kernels[6] = {
            (const void *)kea::rel_attention_kernel<32, 1>, (const void *)kea::rel_attention_kernel<64, 1>,
            (const void *)kea::rel_attention_kernel<128, 1>, (const void *)kea::rel_attention_kernel<32, 2>,
            (const void *)kea::rel_attention_kernel<64, 2>, (const void *)kea::rel_attention_kernel<128, 2>};
        const int attn_smem[6] = {kea::attn_smem_floats<32, 1>() * 4, kea::attn_smem_floats<64, 1>() * 4,
                                  kea::attn_smem_floats<128, 1>() * 4, kea::attn_smem_floats<32, 2>() * 4,
                                  kea::attn_smem_floats<64, 2>() * 4, kea::attn_smem_floats<128, 2>() * 4};
        for (int i = 0; i < 6; ++i)
            if (cudaFuncSetAttribute(attn_kernels[i], cudaFuncAttributeMaxDynamicSharedMemorySize, attn_smem[i]) !=
                cudaSuccess)
                status = KEA_ERR_CUDA;
        const void *gemv_kernels[18] = {
#define KEA_GEMV_MT(W, P) (const void *)kea::lowbit_gemv_kernel<W, P, 1>, (const void *)kea::lowbit_gemv_kernel<W, P, 4>, \
                          (const void *)kea::lowbit_gemv_kernel<W, P, 16>
            KEA_GEMV_MT(1, 1), KEA_GEMV_MT(1, 2), KEA_GEMV_MT(1, 3), KEA_GEMV_MT(2, 1), KEA_GEMV_MT(2, 2), KEA_GEMV_MT(2, 3)
#undef KEA_GEMV_MT
        };
        for (const void *k : gemv_kernels)
            if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kea::kGemvMaxSmem) != cudaSuccess)
                status = KEA_ERR_CUDA;
        const void *reg_kernels[24] = {
#define KEA_REG_P(W, P) (const void *)kea::lowbit_gemm_reg_kernel<W, P, 1, 4, 2>, \
                        (const void *)kea::lowbit_gemm_reg_kernel<W, P, 2, 4, 2>, \
                        (const void *)kea::lowbit_gemm_reg_kernel<W, P, 2, 2, 3>, \
                        (const void *)kea::lowbit_gemm_reg_kernel<W, P, 4, 2, 2>
            KEA_REG_P(1, 1), KEA_REG_P(1, 2), KEA_REG_P(1, 3), KEA_REG_P(2, 1), KEA_REG_P(2, 2), KEA_REG_P(2, 3)
#undef KEA_REG_P
        };
        for (const void *k : reg_kernels)
            if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kRegMaxSmem) != cudaSuccess)
                status = KEA_ERR_CUDA;
    }
    if (status == KEA_OK) {
        void *addr = nullptr;
        if (cudaGetSymbolAddress(&addr, g_noalloc_scratch) != cudaSuccess || !addr) status = KEA_ERR_CUDA;
        st.noalloc_scratch = addr;
    }
    if (status != KEA_OK) cudaGetLastError();
    st.status = status;
    st.sms = sms > 0 ? sms : kSmsB200;
    st.ready = true;
    return status;
}

// ---- configuration ---------------------------------------------------------------------------------------
// Per-stage bytes of the three shared-memory regions (activation tiles, expanded weights, packed codes).
int a_stage_bytes(int tile_m, int parts) { return (tile_m / kea::kBM) * parts * kea::kActTileBytes; }
int b_stage_bytes(int tile_n) { return tile_n * kea::kBK; }
int pk_stage_bytes(int tile_n, int wbits) { return tile_n * 16 * wbits; }
int stage_bytes(int tile_m, int tile_n, int parts, int wbits) {
    return a_stage_bytes(tile_m, parts) + b_stage_bytes(tile_n) + pk_stage_bytes(tile_n, wbits);
}

bool valid_tile_n(int tile_n) { return tile_n == 32 || tile_n == 64 || tile_n == 128 || tile_n == 256; }

// Narrow tiles with one token block and one part keep four partial accumulators (one per K = 32 step).
int accumulators(int tile_m, int tile_n, int parts) { return (tile_n <= 64 && tile_m == kea::kBM && parts == 1) ? 4 : 1; }

uint32_t tmem_columns(int tile_m, int tile_n, int parts) {
    uint32_t need = (uint32_t)((tile_m / kea::kBM) * parts * tile_n * accumulators(tile_m, tile_n, parts)), cols = 32;
    while (cols < need) cols <<= 1;
    return cols;
}

// Split-K receive buffer: [source rank][token block x part][owned channel groups][128 rows] x 16 bytes.
int exchange_bytes(int tile_m, int tile_n, int parts, int splits) {
    if (splits <= 1) return 0;
    const int groups = tile_n / 4, per = ceil_div(groups, splits);
    return splits * (tile_m / kea::kBM) * parts * per * kea::kBM * 16;
}

// The receive buffer gets its own region when it fits beside the stages; otherwise it reuses the stage area.
bool exchange_aliases(int tile_m, int tile_n, int parts, int wbits, int splits, int stages) {
    return stages * stage_bytes(tile_m, tile_n, parts, wbits) + exchange_bytes(tile_m, tile_n, parts, splits) + 1024 >
           kMaxDynSmem;
}

int dyn_smem_bytes(int tile_m, int tile_n, int parts, int wbits, int splits, int stages) {
    const int st = stages * stage_bytes(tile_m, tile_n, parts, wbits);
    const int ex = exchange_bytes(tile_m, tile_n, parts, splits);
    int bytes = exchange_aliases(tile_m, tile_n, parts, wbits, splits, stages) ? std::max(st, ex) : st + ex;
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

// ---- the persistent CTA-pair kernel (gemm_pair_kernel.cuh) ---------------------------------------------------------
// Dynamic shared memory: alignment slack + load slots x (activation box + packed codes) + the B slots + epilogue
// staging + channel constants.
int pair_stage_bytes(int wbits, int parts) { return parts * (int)kea::kPairHalfTile + wbits * kea::kPanelSubBytes; }
int pair_smem_bytes(int wbits, int parts, int stages) {
    return 1024 + stages * pair_stage_bytes(wbits, parts) + kea::kPairBStages * (int)kea::kPairHalfTile +
           (int)kea::kPairStagingBytes + (int)kea::kPairChannelBytes;
}
int pair_max_stages(int wbits, int parts) {
    int s = kea::kPairMaxStages;
    while (s > 2 && pair_smem_bytes(wbits, parts, s) > kPairMaxDynSmem) --s;
    return s;
}
// The pair kernel takes one or two activation parts and whole 256-channel tiles; above this many tokens it replaces
// the per-tile kernel (its 256 x 256 pair tiles keep the shared-memory traffic per MAC at half the per-tile
// kernel's).
constexpr int kPairMinM = 257;
// With two parts the tile's two accumulators fill tensor memory (no overlap of epilogue and MMAs), which costs
// where a few tiles are all the work: below kPairMinTiles2 pair tiles the per-tile kernel measured as fast or faster.
constexpr int kPairMinTiles2 = 32;
// K <= 32768 keeps |acc| <= 127 K below 2^22, where the epilogue's two-operation INT32 -> FP32 conversion is exact.
bool pair_fits(int m, int n, int k, int parts) {
    return parts <= 2 && n % kea::kPairTileN == 0 && m >= kPairMinM && k <= 32768;
}
bool pair_shape(int m, int n, int k, int parts) {
    return pair_fits(m, n, k, parts) &&
           (parts == 1 || ceil_div(m, kea::kPairTileM) * (n / kea::kPairTileN) >= kPairMinTiles2);
}
// Split-K of the pair kernel: when the tiles occupy at most a quarter of the SM pairs and K is long (>= 16
// k-blocks), each tile's K range is cut into slices (>= 4 k-blocks each, at most 8) so that tiles x slices approaches
// the pair count; the slices' INT32 partial sums go through scratch memory and splitk_finish_kernel. Measured
// (B200): N 1024, K 4096, M 512 (8 tiles, 8 slices) 16.5 us against 18.3 unsplit; with 32 tiles or K = 1024 the
// pair kernel's fixed latency (~8 us a launch) dominates and the extra pass made it slower, hence the bounds.
// Returns the slice count (1: unsplit).
int pair_splits(int m, int n, int k, int sms) {
    const int tiles = ceil_div(m, kea::kPairTileM) * (n / kea::kPairTileN), pairs = std::max(1, sms / 2);
    const int kbt = ceil_div(k, kea::kBK);
    if (4 * tiles > pairs || kbt < 16) return 1;
    int s = std::min(std::min(pairs / tiles, kbt / 4), 8);
    if (s < 2) return 1;
    const int kbs = ceil_div(kbt, s);
    return ceil_div(kbt, kbs);   // every slice non-empty
}
size_t pair_workspace_bytes(int m, int n, int k, int parts, int sms) {
    const int s = pair_splits(m, n, k, sms);
    return s > 1 ? (size_t)s * (size_t)parts * (size_t)m * (size_t)n * 4u : 0u;
}

// The weight-stationary pair kernel (gemm_pair_ws_kernel.cuh): one part, K <= 1024, every k-block's expanded weights
// resident: [3 activation slots][kb x 16 KB weights][2 code slots][staging][channel constants].
int pair_ws_smem_bytes(int wbits, int kb) {
    const int stg = round_up(kea::kWsStages * (int)kea::kPairHalfTile + kb * (int)kea::kPairHalfTile +
                             2 * wbits * kea::kPanelSubBytes, 1024);
    return 1024 + stg + (int)kea::kPairStagingBytes + (int)kea::kPairChannelBytes;
}
bool pair_ws_fits(int k, int parts, int wbits) {
    const int kb = ceil_div(k, kea::kBK);
    return parts == 1 && kb <= kea::kWsMaxKb && pair_ws_smem_bytes(wbits, kb) <= kPairMaxDynSmem;
}

KeaGemmConfig pair_config(int wbits, int parts) {
    KeaGemmConfig c{};
    c.tile_m = kea::kPairTileM;
    c.tile_n = kea::kPairTileN;
    c.splits = 1;
    c.stages = pair_max_stages(wbits, parts);
    c.smem_bytes = pair_smem_bytes(wbits, parts, c.stages);
    c.kernel = 1;
    return c;
}

// The M-bucketed split-K dispatch table (B200, 148 SMs).
//  * M <= 128 (one token block): narrow channel tiles, so the grid covers the SMs with little or no split-K
//    (each CTA then reads the whole K of its channels and needs no partial exchange); split K only as far as the
//    one-shot mode needs (<= 8 k-blocks per CTA) and while the tile grid is below the SM count.
//  * 128 < M <= 512: 128-channel tiles, 256 tokens per CTA when one part (the weight expansion serves both
//    token blocks), split K up to the SM count.
//  * larger M: 256 tokens x 256 channels per CTA when the tile count allows (fewest operand bytes per MMA).
// Stacked parts: with P > 1 and P x (M rounded up to 8) <= 128 the parts share one 128-row token tile (part p's
// tokens at rows p * mp ..), so the MMAs, tensor memory and shared memory are those of one part. Needs the 4-D
// activation view (K a multiple of 128).
// Up to 512 tokens the tokens are cut into stacked tiles of mp tokens (P x mp <= 128 rows; mp a multiple of 8).
constexpr int kStackMaxM = 512;
int stack_rows(int m, int parts, int k) {
    return std::min(round_up(std::max(m, 1), 8), (kea::kBM / (8 * std::max(parts, 1))) * 8);
}
bool stackable(int m, int parts, int k) { return parts > 1 && k % kea::kBK == 0 && m <= kStackMaxM; }
// The table's choice: one stacked tile always; above one token block only while unstacked tiles (128 tokens x 128
// channels, P accumulators) would leave half the SMs idle; several stacked tiles run unsplit, so at M <= 128 with
// long K the split unstacked tile wins (measured on the reference's x3 shapes).
bool use_stack(int m, int n, int k, int parts, int sms) {
    if (!stackable(m, parts, k)) return false;
    const bool one_tile = parts * round_up(std::max(m, 1), 8) <= kea::kBM;
    return (m <= kea::kBM || 2 * ceil_div(m, kea::kBM) * ceil_div(n, kea::kPanelN) < sms) &&
           (one_tile || ceil_div(k, kea::kBK) <= 8 || m > kea::kBM);
}

KeaGemmConfig choose_tile(int m, int n, int k, int wbits, int parts_in, int sms, bool allow_stack = true) {
    KeaGemmConfig c{};
    // the tile's footprint: stacked parts act as one
    const bool stacked = allow_stack && use_stack(m, n, k, parts_in, sms);
    const int parts = stacked ? 1 : parts_in;
    const int kb = ceil_div(k, kea::kBK), nt128 = ceil_div(n, kea::kPanelN);
    // token tiles: stacked tiles of mp tokens, else blocks of 128 (or 256) tokens
    const int tok_tiles = stacked ? ceil_div(std::max(m, 1), stack_rows(m, parts_in, k)) : 1;
    int tile_m, tile_n;
    if (stacked && tok_tiles > 1) {
        // several stacked token tiles: split K only for one-shot loading, widen the channel tile until one wave
        tile_m = kea::kBM;
        tile_n = 32;
        while (tile_n < 128 && tok_tiles * ceil_div(n, tile_n) > sms) tile_n *= 2;
    } else if (m <= kea::kBM || stacked) {
        tile_m = kea::kBM;
        tile_n = 32;
        while (tile_n < 128 && tok_tiles * ceil_div(n, tile_n * 2) * 2 >= sms) tile_n *= 2;   // keep >= sms / 2 CTAs
    } else if (m <= 512) {
        tile_m = parts == 1 ? 256 : kea::kBM;
        tile_n = 128;
    } else {
        tile_m = parts == 1 ? 256 : kea::kBM;
        tile_n = (parts == 1 && nt128 % 2 == 0) ? 256 : 128;
        const int tiles256 = ceil_div(n, tile_n) * ceil_div(m, tile_m);
        if (tiles256 < sms && tile_n == 256) tile_n = 128;                  // too few tiles: narrower channels
    }
    const int tiles = (stacked ? tok_tiles : ceil_div(std::max(m, 1), tile_m)) * ceil_div(n, tile_n);
    int splits = 1;
    if (tiles < sms) splits = std::max(1, sms / tiles);
    if (stacked && tok_tiles > 1) splits = 1;
    // One token block: split K only as far as needed for each CTA's K range to arrive in one shot (<= 8 k-blocks);
    // more splits fill more SMs, but the partial exchange costs more than the idle SMs (measured: K = 1024 runs
    // fastest unsplit on 32-64 CTAs, K = 4096 with 4 splits).
    if (m <= kea::kBM || stacked) splits = std::min(splits, ceil_div(kb, 8));
    splits = std::min({splits, kb, kMaxPortableCluster});
    while (splits > 1 && exchange_bytes(tile_m, tile_n, parts, splits) + 1024 > kMaxDynSmem) --splits;
    const int per = ceil_div(kb, splits);
    int stages = std::min(per, max_stages(tile_m, tile_n, parts, wbits));
    c.tile_m = tile_m;
    c.tile_n = tile_n;
    c.splits = splits;
    c.stages = std::max(stages, 1);
    c.smem_bytes = dyn_smem_bytes(tile_m, tile_n, parts, wbits, splits, c.stages);
    c.kernel = 0;
    return c;
}

// ---- the swapped-operand kernel for small M (gemm_swap_kernel.cuh) --------------------------------------------------
// Tokens per token tile: at most 256 (the TMA box's rows) and P x tokens <= 512 (tensor-memory columns), in multiples
// of 16 (the MMA's N step); a shape with more tokens is cut into equal tiles.
int swap_max_tokens(int parts) { return std::min(kea::kSwapMaxTokens, (kea::kSwapMaxRows / parts) / 16 * 16); }
void swap_tokens(int m, int parts, int *mt, int *tiles) {
    *tiles = ceil_div(std::max(m, 1), swap_max_tokens(parts));
    *mt = round_up(ceil_div(std::max(m, 1), *tiles), 16);
}
// A caller's token tile (a multiple of 16 up to swap_max_tokens): tiles of mt tokens, the last one ragged.
bool swap_tokens_forced(int m, int parts, int forced_mt, int *mt, int *tiles) {
    if (forced_mt % 16 || forced_mt < 16 || forced_mt > swap_max_tokens(parts)) return false;
    *mt = forced_mt;
    *tiles = ceil_div(std::max(m, 1), forced_mt);
    return true;
}
// Per stage: the activation box (every part's tokens x 128 k), the expanded weights (128 rows x 128 k), the codes.
int swap_stage_bytes(int rows, int wbits) { return rows * kea::kBK + (int)kea::kSwapWTile + wbits * kea::kPanelSubBytes; }
// Split-K receive buffer: [peer slot (splits - 1)][owned unit][part][4 token quarters][32 channels] x 16 bytes.
int swap_units_per_owner(int mt, int splits) { return ceil_div(4 * (mt / 16), splits); }
int swap_recv_bytes(int mt, int parts, int splits) {
    return splits > 1 ? (splits - 1) * swap_units_per_owner(mt, splits) * parts * kea::kSwapUnitBytes : 0;
}

struct SwapPlan {
    int mt = 0, token_tiles = 0, rows = 0, splits = 1, stages = 1, nacc = 1, smem = 0;
    int recv = 0;                // split-K receive buffer bytes (0 unsplit)
    uint32_t tmem_cols = 32;
};
// The epilogue area (receive buffer, then the epilogue warps' output tiles) starts at the stage area's offset 0: it
// is used only once every MMA of the cluster is done.
constexpr int kSwapStaging = kea::kSwapEpiWarps * kea::kSwapStagingBytes;
int swap_epilogue_bytes(int recv) { return round_up(recv, 1024) + kSwapStaging; }

// The swap kernel's plan for a shape. forced_splits / forced_stages / forced_mt 0 take the table's choice: K split over
// a cluster (<= 8 CTAs) until the channel tiles x token tiles x splits approach the SM count; as many stages as the
// CTA's k-blocks, while two CTAs still fit on an SM; the fewest equal token tiles. False when a forced plan does not
// fit.
bool swap_plan(int m, int n, int k, int wbits, int parts, int sms, int forced_splits, int forced_stages, SwapPlan *out,
               int forced_mt = 0) {
    if (k > 32768) return false;   // |acc| <= 127 K < 2^22: the epilogue's exact two-operation INT32 -> FP32 conversion
    SwapPlan p;
    if (forced_mt) {
        if (!swap_tokens_forced(m, parts, forced_mt, &p.mt, &p.token_tiles)) return false;
    } else {
        swap_tokens(m, parts, &p.mt, &p.token_tiles);
    }
    p.rows = parts * p.mt;
    const int kb = ceil_div(k, kea::kBK);
    const int tiles = ceil_div(n, kea::kPanelN) * p.token_tiles;
    const int stage = swap_stage_bytes(p.rows, wbits);
    int splits = forced_splits ? forced_splits : std::min({kb, kMaxPortableCluster, std::max(1, sms / tiles)});
    // two MMAs per K step (more than 256 stacked rows): the exchange grows with the rows, so split only long K (<= 4)
    if (!forced_splits && p.rows > 256) splits = kb <= 8 ? 1 : std::min(splits, 4);
    if (splits < 1 || splits > kMaxCluster || splits > kb) return false;
    for (;; --splits) {
        if (splits < 1) return false;
        const int recv = swap_recv_bytes(p.mt, parts, splits);
        const int epi = swap_epilogue_bytes(recv);
        if (1024 + epi > kMaxDynSmem) {
            if (forced_splits) return false;
            continue;
        }
        const int nkb = ceil_div(kb, splits);
        int stages = forced_stages;
        if (!stages) {
            stages = std::min(nkb, kea::kSwapStagesMax);
            // two CTAs per SM (programmatic dependent launch overlaps consecutive launches) when that keeps >= 2
            // stages; otherwise as many as fit
            const int two_per_sm = (kSmemPerSm / 2 - 2048 - 1024) / stage;
            if (stages > two_per_sm && two_per_sm >= 2 && std::max(two_per_sm * stage, epi) <= kSmemPerSm / 2 - 3072)
                stages = two_per_sm;
            while (stages > 1 && 1024 + stages * stage > kMaxDynSmem) --stages;
        }
        if (stages < 1 || stages > kea::kSwapStagesMax || 1024 + stages * stage > kMaxDynSmem) return false;
        p.splits = splits;
        p.stages = stages;
        p.recv = recv;
        p.smem = 1024 + std::max(stages * stage, epi);
        break;
    }
    // narrow N (<= 32 stacked rows) is issue-bound: one accumulator per K = 32 step keeps consecutive MMAs independent
    p.nacc = p.rows <= 32 ? 4 : 1;
    const uint32_t need = (uint32_t)(p.nacc * p.rows);
    while (p.tmem_cols < need) p.tmem_cols <<= 1;
    // never more CTAs on an SM than its 512 tensor-memory columns serve (a cluster peer waiting in tcgen05.alloc)
    const int max_ctas = std::max(1, (int)(512 / p.tmem_cols));
    p.smem = std::max(p.smem, kSmemPerSm / (max_ctas + 1) + 1);
    *out = p;
    return true;
}

// Where the table takes the swap kernel (B200, graph-timed cold over the Parakeet shapes against the 128-token-tile
// kernel): one part at M <= 32 (4.7 vs 5.4 us at N 4096, K 1024) and 128 < M <= 256 (its 128-channel tiles serve
// every token at once; 11.4 vs 11.8 us at M 256); several parts once their stacked tokens fill two MMAs (P x M >= 512:
// 10.7 vs 16.6 us at 3 x 256 tokens, N 4096) on wide or deep layers. In between, the tile kernel's 32-channel tiles
// without a partial exchange are faster: at this M the swap kernel's split-K exchange through distributed shared
// memory (~16 B per clock per SM) costs more than the tcgen05 issue slots it saves.
bool swap_shape(int m, int n, int k, int parts) {
    if (m < 1 || k > 32768) return false;
    if (parts == 1) return m <= 32 || (m > 128 && m <= 256);
    return parts * round_up(m, 16) >= 512 && m <= 512 && (n >= 2048 || k >= 4096);
}

KeaGemmConfig swap_config(int m, int n, int k, int wbits, int parts, int sms) {
    SwapPlan p;
    KeaGemmConfig c{};
    if (!swap_plan(m, n, k, wbits, parts, sms, 0, 0, &p)) return c;
    c.tile_m = p.mt;
    c.tile_n = kea::kPanelN;
    c.splits = p.splits;
    c.stages = p.stages;
    c.smem_bytes = p.smem;
    c.kernel = 3;
    return c;
}

// The CUDA-core kernel: 8 channels per CTA (32 K slices per channel) spreads even 1024-channel layers over the SMs.
// 16 (fewer, longer slices) measured faster for small weights (N x K <= 1M: the whole job is a few CTAs per SM) and
// for wide layers (N > 3072) with several activation rows, unless the rows are the tokens of one 2-bit part (its
// words carry half the codes, so its slices are already twice as long). The table takes the kernel up to
// kGemvTableRows activation rows (tokens x parts), where it beat the tensor-core kernel on every Parakeet shape;
// from 6 rows on the tensor-core kernel is as fast or faster.
constexpr int kGemvTableRows = 4;
int gemv_channels(int n, int k, int wbits, int m, int parts) {
    if ((long long)n * k <= (1LL << 20)) return 16;
    if (n > 3072 && m * parts >= 2 && (wbits == 1 || parts > 1)) return 16;
    return 8;
}
bool gemv_fits(int m, int parts, int ch) {
    return m >= 1 && m <= kea::kGemvMaxM && kea::gemv_smem_bytes(m * parts, ch) <= kea::kGemvMaxSmem;
}

// One part on a narrow layer (512 < N <= 1024, K <= 4096: the measured range) just above the pair kernel's M threshold: its 256 x 256 tiles are too few
// to fill the SMs (8-16 pairs of 74), and the per-tile kernel with 128-token tiles and K split over a cluster of up to
// 4 fills them instead. Measured (B200, graph-timed cold, one part): N 1024, K 4096, M 300-512: 11.0-11.5 us
// (128 x 128 tiles, 4 slices) against 16.0-16.5 for the pair kernel; M 768-1024: 15.3 against 18.8-19.1 (2 slices);
// N 1024, K 1024, M 300-512: 6.3-6.8 (128 x 64 tiles, 2 slices) against 8.4-8.5. From M 768 at K 1024 and M 1536 at
// K 4096 the pair kernel is as fast or faster.
bool narrow_mid_m(int m, int n, int k, int parts) {
    return parts == 1 && n > 512 && n <= 1024 && k <= 4096 && m >= kPairMinM && m <= (k >= 2048 ? 1024 : 512);
}
KeaGemmConfig narrow_mid_config(int m, int n, int k, int wbits, int sms) {
    KeaGemmConfig c{};
    const int kb = ceil_div(k, kea::kBK);
    c.tile_m = kea::kBM;
    c.tile_n = k >= 2048 ? 128 : 64;
    const int tiles = ceil_div(m, kea::kBM) * ceil_div(n, c.tile_n);
    int splits = 1;
    while (splits < 4 && tiles * splits * 2 <= sms && splits * 2 <= kb) splits *= 2;
    c.splits = splits;
    c.stages = std::max(1, std::min({4, ceil_div(kb, splits), max_stages(c.tile_m, c.tile_n, 1, wbits)}));
    c.smem_bytes = dyn_smem_bytes(c.tile_m, c.tile_n, 1, wbits, splits, c.stages);
    c.kernel = 0;
    return c;
}

// The full table: the CUDA-core kernel for M x parts <= 4, the swap kernel up to 256 tokens, the pair kernel where its
// shape rule holds (except narrow layers just above its M threshold), else the per-tile kernel's entry.
// The register-operand kernel's tiles for a shape: tile_n channels x tile_m activation rows (tokens x parts) per CTA,
// splits K-slices among its 8 warps. Measured (B200, graph-timed, 4 rotating weight sets): about 256 CTAs is best,
// and of two tiles with the same count the one with more channels (fewer re-reads of the activation rows); 16 rows x
// 32 channels is the base tile; where it would exceed ~320 CTAs, 16 x 64 on N >= 2048 (N 2048, M 125 in the clip:
// 3.012 against 3.023 ms for 32 x 32) and 32 x 32 below; 32 x 16 for 16 rows or fewer where the base tile would give
// fewer than ~160.
KeaGemmConfig reg_config(int m, int n, int k, int parts, int sms) {
    (void)k;
    (void)sms;
    KeaGemmConfig c{};
    c.kernel = 4;
    c.tile_m = 16;
    c.tile_n = 32;
    c.splits = 8;
    c.stages = 0;
    const long long rows = (long long)m * parts;
    const long long ctas = (long long)ceil_div(n, 32) * ceil_div(m, 16 / parts);
    if (ctas > 320) {
        if (n >= 2048) c.tile_n = 64;
        else c.tile_m = 32;
    } else if (ctas < 160 && rows <= 16) {
        c.tile_m = 32;
        c.tile_n = 16;
    }
    c.smem_bytes = kea::reg_smem_bytes(c.splits, c.tile_m, c.tile_n);
    return c;
}

// Where the table takes the register kernel (activation rows = tokens x parts, above the CUDA-core kernel's 4).
// Measured against the tcgen05 table's choice (graph-timed, without / with programmatic dependent launch): faster
// while rows x N <= 160 K at up to 256 rows (N 1024, K 1024, M 125: 4.3 / 3.2 us against 6.7 / 4.6; N 4096,
// K 1024, M 16: 3.8 / 2.8 against 6.6 / 4.9; three parts, N 1024, K 1024, M 38: 3.9 / 2.8 against 6.2 / 4.0) and on
// narrow layers with long K (N 1024, K 4096, M 125: 6.9 / 5.8 against 7.8 / 6.7; three parts at M 126: 12.9 / 12.0
// against 14.2 / 13.0) up to 128 rows, or 400 rows of three parts. N 2048, K 1024, M 125 (rows x N = 256 K) is
// about even in a GEMM chain (5.9 / 4.9 us against 6.7 / 4.6) but faster in the config-2 clip, where the GEMM follows
// its quantizer (whole clip 3.061 -> 3.012 ms), so rows x N <= 256 K is taken on N >= 2048, K <= 1024 too. Wider
// layers at M 125 (N 3072-4096) stay on the tcgen05 kernels (the clip with them here: 3.108 ms): their activation
// rows are re-read by N / 64 CTAs.
bool reg_shape(int m, int n, int k, int parts) {
    const long long rows = (long long)m * parts;
    if (rows <= 256 && rows * n <= 160LL * 1024) return true;
    if (n >= 2048 && k <= 1024 && rows * n <= 256LL * 1024) return true;
    return n <= 1024 && k >= 4096 && (rows <= 128 || (parts == 3 && rows <= 400));
}

KeaGemmConfig choose(int m, int n, int k, int wbits, int parts, int sms, bool allow_reg = true) {
    KeaGemmConfig c = choose_tile(m, n, k, wbits, parts, sms);
    if (swap_shape(m, n, k, parts)) {
        const KeaGemmConfig s = swap_config(m, n, k, wbits, parts, sms);
        if (s.kernel == 3) c = s;
    }
    if (pair_shape(m, n, k, parts)) c = narrow_mid_m(m, n, k, parts) ? narrow_mid_config(m, n, k, wbits, sms)
                                                                     : pair_config(wbits, parts);
    if (m * parts <= kGemvTableRows && gemv_fits(m, parts, gemv_channels(n, k, wbits, m, parts))) {
        c.kernel = 2;
        c.tile_m = m;
        c.tile_n = gemv_channels(n, k, wbits, m, parts);
        c.splits = 1;
        c.stages = 1;
        c.smem_bytes = kea::gemv_smem_bytes(m * parts, c.tile_n);
    } else if (allow_reg && reg_shape(m, n, k, parts)) {
        c = reg_config(m, n, k, parts, sms);
    }
    return c;
}

int check_config(const KeaGemmConfig &c, int n, int k, int parts, int wbits) {
    // parts here is the tile footprint: 1 for stacked parts
    const int kb = ceil_div(k, kea::kBK), nt = ceil_div(n, kea::kPanelN);
    if (c.tile_m != 128 && c.tile_m != 256) return KEA_ERR_UNSUPPORTED;
    if (!valid_tile_n(c.tile_n)) return KEA_ERR_UNSUPPORTED;
    if (c.tile_n == 256 && nt % 2) return KEA_ERR_UNSUPPORTED;   // the second panel tile must exist
    if ((c.tile_m / kea::kBM) * parts * c.tile_n > 512) return KEA_ERR_UNSUPPORTED;   // TMEM columns
    if (c.splits < 1 || c.splits > kMaxCluster || c.splits > kb) return KEA_ERR_UNSUPPORTED;
    if (c.stages < 1 || c.stages > kea::kMaxStages) return KEA_ERR_UNSUPPORTED;
    if (c.smem_bytes > kMaxDynSmem) return KEA_ERR_UNSUPPORTED;
    (void)wbits;
    return KEA_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// A launch configuration on `stream` with `dyn` bytes of dynamic shared memory, optionally with programmatic
// dependent launch (the kernel may start while the previous one finishes; it waits in griddepcontrol.wait).
cudaLaunchConfig_t launch_config(dim3 grid, size_t dyn, void *stream, cudaLaunchAttribute *attr, int pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kea::kQuantThreads, 1, 1);
    cfg.dynamicSmemBytes = dyn;
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    cfg.numAttrs = 0;
    if (pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 1;
    }
    return cfg;
}

// Launches the CUDA-core kernel for M <= 16 (any wbits / parts / layout the per-tile kernel takes).
template <int W, int P>
cudaError_t launch_gemv_p(cudaLaunchConfig_t *cfg, const kea::GemvArgs &a) {
    if (a.M <= 1) return cudaLaunchKernelEx(cfg, kea::lowbit_gemv_kernel<W, P, 1>, a);
    if (a.M <= 4) return cudaLaunchKernelEx(cfg, kea::lowbit_gemv_kernel<W, P, 4>, a);
    return cudaLaunchKernelEx(cfg, kea::lowbit_gemv_kernel<W, P, 16>, a);
}

int launch_gemv(const KeaGemmDesc *d, const KeaGemmConfig &c, void *stream) {
    kea::GemvArgs a{};
    a.q = d->q;
    a.q_stride = d->parts > 1 ? d->q_part_stride : 0;
    a.ldq = d->ldq;
    a.qs = d->qs;
    a.qs_stride = d->qs_part_stride;
    a.panels = d->panels;
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
    a.kb_total = ceil_div(d->k, kea::kBK);
    a.ch = c.tile_n;
    a.flags = d->flags & (KEA_FLAG_SILU | KEA_FLAG_ORDER1);
    a.err = d->error_word;
    a.res = d->residual;
    a.ld_res = d->ld_residual;
    a.res_scale = d->residual_scale;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(d->n, c.tile_n), 1, 1);
    cfg.blockDim = dim3(kea::kGemvThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)kea::gemv_smem_bytes(d->m * d->parts, c.tile_n);
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    if (d->flags & KEA_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 1;
    }
    cudaError_t e;
    switch (d->wbits * 4 + d->parts) {
        case 5: e = launch_gemv_p<1, 1>(&cfg, a); break;
        case 6: e = launch_gemv_p<1, 2>(&cfg, a); break;
        case 7: e = launch_gemv_p<1, 3>(&cfg, a); break;
        case 9: e = launch_gemv_p<2, 1>(&cfg, a); break;
        case 10: e = launch_gemv_p<2, 2>(&cfg, a); break;
        default: e = launch_gemv_p<2, 3>(&cfg, a); break;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return KEA_ERR_CUDA;
    }
    return KEA_OK;
}

// The register-operand kernel (warp MMAs, weights expanded in registers): `cn` channels x `rows` activation rows
// (tokens x parts) per CTA, its 8 warps cut into `ks` K-slices x 8 / ks channel groups of 16 x cg channels.
struct RegPlan {
    int cg = 0, rg = 0, ks = 0, cn = 0, rows = 0, tt = 0;
};

// The instantiated warp tiles (cg channel groups x rg row groups): 16 x cg channels x 8 x rg rows per warp.
bool reg_tile_ok(int cg, int rg) { return (cg == 1 && rg == 4) || (cg == 2 && (rg == 4 || rg == 2)) || (cg == 4 && rg == 2); }

bool reg_plan(int m, int parts, int cn, int rows, int ks, RegPlan *p) {
    if (ks != 1 && ks != 2 && ks != 4 && ks != 8) return false;
    if (cn != 16 && cn != 32 && cn != 64 && cn != 128) return false;   // divides the 128-row panel tile
    if (rows != 16 && rows != 32) return false;
    const int cw = kea::kRegWarps / ks;
    if (cn % (16 * cw)) return false;
    const int cg = cn / (16 * cw), rg = rows / 8;
    if (!reg_tile_ok(cg, rg) || rows / parts < 1) return false;
    if (ceil_div(m, rows / parts) > 65535) return false;   // token tiles are the grid's y dimension
    p->cg = cg;
    p->rg = rg;
    p->ks = ks;
    p->cn = cn;
    p->rows = rows;
    p->tt = rows / parts;
    return true;
}

template <int W, int P>
cudaError_t launch_reg_p(cudaLaunchConfig_t *cfg, const kea::RegArgs &a, const RegPlan &p) {
    if (p.cg == 1) return cudaLaunchKernelEx(cfg, kea::lowbit_gemm_reg_kernel<W, P, 1, 4, 2>, a);
    if (p.cg == 4) return cudaLaunchKernelEx(cfg, kea::lowbit_gemm_reg_kernel<W, P, 4, 2, 2>, a);
    if (p.rg == 2) return cudaLaunchKernelEx(cfg, kea::lowbit_gemm_reg_kernel<W, P, 2, 2, 3>, a);
    return cudaLaunchKernelEx(cfg, kea::lowbit_gemm_reg_kernel<W, P, 2, 4, 2>, a);
}

int launch_reg(const KeaGemmDesc *d, const RegPlan &p, void *stream) {
    kea::RegArgs a{};
    a.q = d->q;
    a.q_stride = d->parts > 1 ? d->q_part_stride : 0;
    a.ldq = d->ldq;
    a.qs = d->qs;
    a.qs_stride = d->qs_part_stride;
    a.panels = d->panels;
    a.alpha = d->alpha;
    a.bias = d->bias;
    a.y = d->y;
    a.ldy = d->ldy;
    a.y_f16 = d->y_dtype == KEA_OUT_F16;
    a.acc = d->acc;
    a.ld_acc = d->ld_acc;
    a.acc_stride = d->acc_part_stride;
    a.res = d->residual;
    a.ld_res = d->ld_residual;
    a.res_scale = d->residual_scale;
    a.M = d->m;
    a.N = d->n;
    a.K = d->k;
    a.kb_total = ceil_div(d->k, kea::kBK);
    a.ks = p.ks;
    a.tt = p.tt;
    a.flags = d->flags & (KEA_FLAG_SILU | KEA_FLAG_ORDER1);
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(d->n, p.cn), (unsigned)ceil_div(d->m, p.tt), 1);
    cfg.blockDim = dim3(kea::kRegThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)kea::reg_smem_bytes(p.ks, p.rows, p.cn);
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    if (d->flags & KEA_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 1;
    }
    cudaError_t e;
    switch (d->wbits * 4 + d->parts) {
        case 5: e = launch_reg_p<1, 1>(&cfg, a, p); break;
        case 6: e = launch_reg_p<1, 2>(&cfg, a, p); break;
        case 7: e = launch_reg_p<1, 3>(&cfg, a, p); break;
        case 9: e = launch_reg_p<2, 1>(&cfg, a, p); break;
        case 10: e = launch_reg_p<2, 2>(&cfg, a, p); break;
        default: e = launch_reg_p<2, 3>(&cfg, a, p); break;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return KEA_ERR_CUDA;
    }
    return KEA_OK;
}

// Launches the persistent CTA-pair kernel. KEA_ERR_UNSUPPORTED when an operand's alignment or stride rules it out
// (the caller then runs the per-tile kernel); other codes are final.
// The pair kernel's epilogue stores 16-byte vectors and TMA boxes: its outputs and channel constants must be aligned.
bool pair_operands_ok(const KeaGemmDesc *d) {
    const int esize = d->y_dtype == KEA_OUT_F16 ? 2 : 4;
    return aligned16(d->y) && (d->ldy * esize) % 16 == 0 && aligned16(d->alpha) && (!d->bias || aligned16(d->bias)) &&
           (!d->acc || (aligned16(d->acc) && d->ld_acc % 4 == 0 && (d->parts == 1 || d->acc_part_stride % 4 == 0))) &&
           (!d->residual || (aligned16(d->residual) && d->ld_residual % 4 == 0));
}

int launch_pair(const KeaGemmDesc *d, const KeaGemmConfig &c, int sms, void *stream) {
    const int esize = d->y_dtype == KEA_OUT_F16 ? 2 : 4;
    if (!pair_operands_ok(d)) return KEA_ERR_UNSUPPORTED;
    // Activations: 3-D (k, row, part) with 128 x 128 x 1 boxes in the 128-byte swizzle; columns >= k and rows >= m
    // read as 0.
    CUtensorMap qmap, ymap;
    {
        const long long pstride = d->parts > 1 ? d->q_part_stride : (long long)d->m * d->ldq;
        const cuuint64_t dims[3] = {(cuuint64_t)d->k, (cuuint64_t)d->m, (cuuint64_t)d->parts};
        const cuuint64_t strides[2] = {(cuuint64_t)d->ldq, (cuuint64_t)pstride};
        const cuuint32_t box[3] = {(cuuint32_t)kea::kBK, (cuuint32_t)kea::kBM, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        if (g_encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(d->q), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return KEA_ERR_CUDA;
    }
    // Output: 32 rows x 64 bytes per store (32 FP16 or 16 FP32 channels), 64-byte swizzle; rows >= m are not written.
    {
        const cuuint64_t dims[2] = {(cuuint64_t)d->n, (cuuint64_t)d->m};
        const cuuint64_t strides[1] = {(cuuint64_t)(d->ldy * esize)};
        const cuuint32_t box[2] = {(cuuint32_t)(64 / esize), 32};
        const cuuint32_t estr[2] = {1, 1};
        if (g_encode(&ymap, esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, d->y, dims,
                     strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return KEA_ERR_UNSUPPORTED;
    }
    kea::PairArgs a{};
    a.panels = d->panels;
    a.qs = d->qs;
    a.qs_stride = d->qs_part_stride;
    a.alpha = d->alpha;
    a.bias = d->bias;
    a.acc = d->acc;
    a.ld_acc = d->ld_acc;
    a.acc_stride = d->acc_part_stride;
    a.M = d->m;
    a.N = d->n;
    a.K = d->k;
    a.kb_total = ceil_div(d->k, kea::kBK);
    a.n_tiles = d->n / kea::kPairTileN;
    a.m_tiles = ceil_div(d->m, kea::kPairTileM);
    a.tiles = a.n_tiles * a.m_tiles;
    a.flags = d->flags & (KEA_FLAG_SILU | KEA_FLAG_ORDER1);
    a.res = d->residual;
    a.ld_res = d->ld_residual;
    a.res_scale = d->residual_scale;
    a.pdl = (d->flags & KEA_FLAG_PDL) ? 1 : 0;
    a.y_f16 = esize == 2;
    a.stages = c.stages;
    a.err = d->error_word;
    // split-K through the caller's scratch, when the shape wants it and the workspace holds it
    const int splits = pair_splits(d->m, d->n, d->k, sms);
    const size_t ws_need = pair_workspace_bytes(d->m, d->n, d->k, d->parts, sms);
    const bool split = splits > 1 && d->workspace && aligned16(d->workspace) &&
                       (size_t)std::max<int64_t>(d->workspace_bytes, 0) >= ws_need;
    a.splits = split ? splits : 1;
    a.kbs = split ? ceil_div(a.kb_total, splits) : a.kb_total;
    a.items = a.tiles * a.splits;
    a.ws = split ? static_cast<int *>(d->workspace) : nullptr;
    if (split) {   // the finish kernel writes y, acc and the residual sum
        a.acc = nullptr;
        a.res = nullptr;
    }
    const int pairs = std::min(a.items, std::max(1, sms / 2));
    // Weight-stationary (one part, K <= 1024, unsplit): runs of tiles keep a channel tile's expanded weights.
    const bool ws = !split && !(d->flags & KEA_FLAG_NO_RESIDENT_WEIGHTS) && pair_ws_fits(d->k, d->parts, d->wbits);

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
    cfg.blockDim = dim3(kea::kPairThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)(ws ? pair_ws_smem_bytes(d->wbits, a.kb_total) : c.smem_bytes);
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attrs[2];
    unsigned na = 0;
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = 2;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
    if (d->flags & KEA_FLAG_PDL) {
        attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attrs[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    cfg.attrs = attrs;
    cfg.numAttrs = na;
    cudaError_t e;
    if (ws)
        e = d->wbits == 1 ? cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_pair_ws_kernel<1>, qmap, ymap, a)
                          : cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_pair_ws_kernel<2>, qmap, ymap, a);
    else switch (d->wbits * 4 + d->parts) {
        case 5: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_pair_kernel<1, 1>, qmap, ymap, a); break;
        case 6: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_pair_kernel<1, 2>, qmap, ymap, a); break;
        case 9: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_pair_kernel<2, 1>, qmap, ymap, a); break;
        default: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_pair_kernel<2, 2>, qmap, ymap, a); break;
    }
    if (e == cudaSuccess && split) {
        kea::SplitFinishArgs f{};
        f.ws = a.ws;
        f.splits = splits;
        f.parts = d->parts;
        f.M = d->m;
        f.N = d->n;
        f.qs = d->qs;
        f.qs_stride = d->qs_part_stride;
        f.alpha = d->alpha;
        f.bias = d->bias;
        f.y = d->y;
        f.ldy = d->ldy;
        f.y_f16 = esize == 2;
        f.acc = d->acc;
        f.ld_acc = d->ld_acc;
        f.acc_stride = d->acc_part_stride;
        f.res = d->residual;
        f.ld_res = d->ld_residual;
        f.res_scale = d->residual_scale;
        f.flags = d->flags & (KEA_FLAG_SILU | KEA_FLAG_ORDER1);
        cudaLaunchConfig_t fc = {};
        const long long threads = (long long)d->m * (d->n / 4);
        fc.gridDim = dim3((unsigned)((threads + 255) / 256), 1, 1);
        fc.blockDim = dim3(256, 1, 1);
        fc.stream = (cudaStream_t)stream;
        cudaLaunchAttribute fattr[1];
        fc.attrs = fattr;
        if (d->flags & KEA_FLAG_PDL) {   // its CTAs wait (griddepcontrol.wait) for the partial sums
            fattr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            fattr[0].val.programmaticStreamSerializationAllowed = 1;
            fc.numAttrs = 1;
        }
        e = cudaLaunchKernelEx(&fc, kea::splitk_finish_kernel, f);
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return KEA_ERR_CUDA;
    }
    return KEA_OK;
}

// Argument checks of kea_lowbit_gemm (and its no-allocation variant): KEA_OK for a valid descriptor (m == 0 included).
int validate_gemm(const KeaGemmDesc *d) {
    if (!d) return KEA_ERR_INVALID_VALUE;
    if (d->m < 0 || d->n < 1 || d->k < 1 || d->parts < 1 || d->parts > 3 || (d->wbits != 1 && d->wbits != 2) ||
        (d->y_dtype != KEA_OUT_F32 && d->y_dtype != KEA_OUT_F16))
        return KEA_ERR_INVALID_VALUE;
    if (d->m == 0) return KEA_OK;
    if (!d->q || !d->qs || !d->panels || !d->alpha || !d->y || d->ldy < d->n || d->ldq < d->k) return KEA_ERR_INVALID_VALUE;
    if (d->acc && (d->ld_acc < d->n || (d->parts > 1 && d->acc_part_stride < (int64_t)d->m * d->ld_acc)))
        return KEA_ERR_INVALID_VALUE;
    if (d->residual && (d->y_dtype != KEA_OUT_F32 || d->ld_residual < d->n)) return KEA_ERR_INVALID_VALUE;
    if (!aligned16(d->q) || d->ldq % 16 || !aligned16(d->panels)) return KEA_ERR_ALIGNMENT;
    if (d->parts > 1 && (d->q_part_stride % 16 || d->q_part_stride < (int64_t)d->m * d->ldq)) return KEA_ERR_ALIGNMENT;
    if (d->flags & ~(KEA_FLAG_SILU | KEA_FLAG_ORDER1 | KEA_FLAG_PDL | KEA_FLAG_NO_PAIR | KEA_FLAG_FORCE_PAIR |
                     KEA_FLAG_FORCE_SWAP | KEA_FLAG_NO_SWAP | KEA_FLAG_TEST_STALL | KEA_FLAG_NO_RESIDENT_WEIGHTS |
                     KEA_FLAG_FORCE_REG | KEA_FLAG_NO_REG))
        return KEA_ERR_INVALID_VALUE;
    if ((d->flags & KEA_FLAG_NO_PAIR) && (d->flags & KEA_FLAG_FORCE_PAIR)) return KEA_ERR_INVALID_VALUE;
    // forced swap: tile_m is its token tile (0, or a multiple of 16), tile_n unused
    if ((d->flags & KEA_FLAG_FORCE_SWAP) &&
        (d->tile_m % 16 || d->tile_m < 0 || d->tile_n || (d->flags & (KEA_FLAG_NO_SWAP | KEA_FLAG_FORCE_PAIR))))
        return KEA_ERR_INVALID_VALUE;
    if ((d->flags & KEA_FLAG_TEST_STALL) && !(d->flags & KEA_FLAG_FORCE_SWAP)) return KEA_ERR_INVALID_VALUE;
    // forced register-operand kernel: tile_n channels and tile_m rows per CTA, splits K-slices (0: the table's)
    if ((d->flags & KEA_FLAG_FORCE_REG) &&
        (d->stages || (d->flags & (KEA_FLAG_NO_REG | KEA_FLAG_FORCE_SWAP | KEA_FLAG_FORCE_PAIR))))
        return KEA_ERR_INVALID_VALUE;
    if (d->wait_clocks < 0) return KEA_ERR_INVALID_VALUE;
    return KEA_OK;
}

// ---- routing: the one decision of which kernel runs a descriptor (the launch, the no-allocation scratch check) ----
enum Route { kRouteGemv, kRoutePair, kRouteSwap, kRouteTile, kRouteReg };

int route_gemm(const KeaGemmDesc *d, int sms, Route *route, KeaGemmConfig *c, SwapPlan *sp, RegPlan *rp) {
    const bool forced = d->tile_m || d->tile_n || d->splits || d->stages;
    if (d->flags & KEA_FLAG_FORCE_REG) {   // channels / rows / K-slices (0: the table's) apply to the register kernel
        const KeaGemmConfig t = reg_config(d->m, d->n, d->k, d->parts, sms);
        if (!reg_plan(d->m, d->parts, d->tile_n ? d->tile_n : t.tile_n, d->tile_m ? d->tile_m : t.tile_m,
                      d->splits ? d->splits : t.splits, rp))
            return KEA_ERR_UNSUPPORTED;
        *route = kRouteReg;
        return KEA_OK;
    }
    if (d->flags & KEA_FLAG_FORCE_SWAP) {   // token tile / splits / stages (0: the table's) apply to the swap kernel
        if (!swap_plan(d->m, d->n, d->k, d->wbits, d->parts, sms, d->splits, d->stages, sp, d->tile_m))
            return KEA_ERR_UNSUPPORTED;
        *route = kRouteSwap;
        return KEA_OK;
    }
    *c = choose(d->m, d->n, d->k, d->wbits, d->parts, sms);
    if (c->kernel == 2 && !forced) {
        *route = kRouteGemv;
        return KEA_OK;
    }
    if (forced && d->tile_m >= 1 && d->tile_m <= kea::kGemvMaxM) {   // the CUDA-core kernel, forced
        if ((d->tile_n != 8 && d->tile_n != 16 && d->tile_n != 32) || !gemv_fits(d->m, d->parts, d->tile_n) ||
            d->splits > 1 || d->stages > 1)
            return KEA_ERR_UNSUPPORTED;
        c->kernel = 2;
        c->tile_m = d->m;
        c->tile_n = d->tile_n;
        *route = kRouteGemv;
        return KEA_OK;
    }
    if (!forced && (d->flags & KEA_FLAG_FORCE_PAIR) && pair_fits(d->m, d->n, d->k, d->parts))
        *c = pair_config(d->wbits, d->parts);
    if (!forced && c->kernel == 1 && !(d->flags & KEA_FLAG_NO_PAIR) && pair_operands_ok(d)) {
        *route = kRoutePair;
        return KEA_OK;
    }
    if (!forced && c->kernel == 4 && !(d->flags & KEA_FLAG_NO_REG) &&
        reg_plan(d->m, d->parts, c->tile_n, c->tile_m, c->splits, rp)) {
        *route = kRouteReg;
        return KEA_OK;
    }
    if (!forced && c->kernel == 4)   // kept off the register kernel: the tcgen05 table's choice for the shape
        *c = choose(d->m, d->n, d->k, d->wbits, d->parts, sms, false);
    if (!forced && c->kernel == 3 && !(d->flags & KEA_FLAG_NO_SWAP) &&
        swap_plan(d->m, d->n, d->k, d->wbits, d->parts, sms, 0, 0, sp)) {
        *route = kRouteSwap;
        return KEA_OK;
    }
    *route = kRouteTile;
    return KEA_OK;
}

// The split-K scratch the routed launch of this descriptor writes (the pair kernel's slices), 0 for none.
size_t routed_scratch_bytes(const KeaGemmDesc *d, int sms) {
    Route r;
    KeaGemmConfig c{};
    SwapPlan sp;
    RegPlan rp;
    if (route_gemm(d, sms, &r, &c, &sp, &rp) != KEA_OK || r != kRoutePair) return 0;
    return pair_workspace_bytes(d->m, d->n, d->k, d->parts, sms);
}

int launch_swap(const KeaGemmDesc *d, const SwapPlan &p, void *stream) {
    const int kb_total = ceil_div(d->k, kea::kBK);
    const bool q4d = d->k % kea::kBK == 0;
    const long long pstride = d->parts > 1 ? d->q_part_stride : (long long)d->m * d->ldq;
    // Activations: (k in block, row, part, k-block) with one box per stage of 128 k x mt rows x every part, landing
    // as [part][row][128 bytes] (part p's tokens at rows p * mt); or, when K is not a multiple of 128, (k, row, part)
    // with one 128 x mt box per part whose columns >= k read as zero. 128-byte swizzle; rows >= m read as zero.
    CUtensorMap qmap;
    CUresult r;
    if (q4d) {
        const cuuint64_t dims[4] = {(cuuint64_t)kea::kBK, (cuuint64_t)d->m, (cuuint64_t)d->parts, (cuuint64_t)kb_total};
        const cuuint64_t strides[3] = {(cuuint64_t)d->ldq, (cuuint64_t)std::max<long long>(pstride, 16), (cuuint64_t)kea::kBK};
        const cuuint32_t box[4] = {(cuuint32_t)kea::kBK, (cuuint32_t)p.mt, (cuuint32_t)d->parts, 1};
        const cuuint32_t estr[4] = {1, 1, 1, 1};
        r = g_encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t *>(d->q), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const cuuint64_t dims[3] = {(cuuint64_t)d->k, (cuuint64_t)d->m, (cuuint64_t)d->parts};
        const cuuint64_t strides[2] = {(cuuint64_t)d->ldq, (cuuint64_t)std::max<long long>(pstride, 16)};
        const cuuint32_t box[3] = {(cuuint32_t)kea::kBK, (cuuint32_t)p.mt, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        r = g_encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(d->q), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return KEA_ERR_CUDA;
    // Output: TMA box stores of 32 channels x 16 tokens (no swizzle) when y's base and row stride allow them.
    const int esize = d->y_dtype == KEA_OUT_F16 ? 2 : 4;
    CUtensorMap ymap;
    std::memset(&ymap, 0, sizeof(ymap));
    bool tma_store = aligned16(d->y) && (d->ldy * esize) % 16 == 0;
    if (tma_store) {
        const cuuint64_t ydims[2] = {(cuuint64_t)d->n, (cuuint64_t)d->m};
        const cuuint64_t ystrides[1] = {(cuuint64_t)(d->ldy * esize)};
        const cuuint32_t ybox[2] = {32, 16};
        const cuuint32_t yestr[2] = {1, 1};
        if (g_encode(&ymap, esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, d->y, ydims,
                     ystrides, ybox, yestr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            tma_store = false;
    }
    kea::SwapArgs a{};
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
    a.res = d->residual;
    a.ld_res = d->ld_residual;
    a.res_scale = d->residual_scale;
    a.M = d->m;
    a.N = d->n;
    a.K = d->k;
    a.kb_total = kb_total;
    a.splits = p.splits;
    a.stages = p.stages;
    a.mt = p.mt;
    a.rows = p.rows;
    a.nacc = p.nacc;
    a.tmem_cols = p.tmem_cols;
    a.a_stage = (uint32_t)(p.rows * kea::kBK);
    a.w_region = (uint32_t)p.stages * a.a_stage;
    a.pk_region = a.w_region + (uint32_t)p.stages * kea::kSwapWTile;
    a.epi_off = 0;
    a.stg_off = (uint32_t)round_up(p.recv, 1024);
    a.epi_alias = p.splits > 1 ? 1 : 0;
    a.tma_store = tma_store ? 1 : 0;
    a.units_per_owner = swap_units_per_owner(p.mt, p.splits);
    a.q4d = q4d ? 1 : 0;
    a.flags = d->flags & (KEA_FLAG_SILU | KEA_FLAG_ORDER1);
    a.pdl = (d->flags & KEA_FLAG_PDL) ? 1 : 0;
    a.stall = (d->flags & KEA_FLAG_TEST_STALL) ? 1 : 0;
    a.wait_clocks = d->wait_clocks > 0 ? d->wait_clocks : kea::kWaitBudget;
    a.err = d->error_word;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(d->n, kea::kPanelN), (unsigned)p.token_tiles, (unsigned)p.splits);
    cfg.blockDim = dim3(kea::kSwapThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)p.smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attrs[2];
    unsigned na = 0;
    if (p.splits > 1) {
        attrs[na].id = cudaLaunchAttributeClusterDimension;
        attrs[na].val.clusterDim.x = 1;
        attrs[na].val.clusterDim.y = 1;
        attrs[na].val.clusterDim.z = (unsigned)p.splits;
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
        case 5: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_swap_kernel<1, 1>, qmap, ymap, a); break;
        case 6: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_swap_kernel<1, 2>, qmap, ymap, a); break;
        case 7: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_swap_kernel<1, 3>, qmap, ymap, a); break;
        case 9: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_swap_kernel<2, 1>, qmap, ymap, a); break;
        case 10: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_swap_kernel<2, 2>, qmap, ymap, a); break;
        default: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_swap_kernel<2, 3>, qmap, ymap, a); break;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return KEA_ERR_CUDA;
    }
    return KEA_OK;
}

}  // namespace

// Two key groups per CTA when the grid is small (under two CTAs per SM): each CTA's chain of key blocks halves.
template <int DK>
cudaError_t launch_rel_attention(cudaLaunchConfig_t *cfg, const kea::RelAttnArgs &a, int sms) {
    const long long ctas = (long long)cfg->gridDim.x * cfg->gridDim.y * cfg->gridDim.z;
    if (ctas < 2LL * sms) {
        cfg->blockDim = dim3(2 * kea::kAttnThreads, 1, 1);
        cfg->dynamicSmemBytes = (size_t)kea::attn_smem_floats<DK, 2>() * sizeof(float);
        return cudaLaunchKernelEx(cfg, kea::rel_attention_kernel<DK, 2>, a);
    }
    cfg->dynamicSmemBytes = (size_t)kea::attn_smem_floats<DK, 1>() * sizeof(float);
    return cudaLaunchKernelEx(cfg, kea::rel_attention_kernel<DK, 1>, a);
}

template <int KW>
cudaError_t launch_glu_dw(cudaLaunchConfig_t *cfg, const kea::ConvArgs &a) {
    return cudaLaunchKernelEx(cfg, kea::glu_depthwise_kernel<KW>, a);
}
template <int KW>
cudaError_t launch_glu_dw_quant(cudaLaunchConfig_t *cfg, const kea::ConvQuantArgs &a, int frames) {
    return frames == 4 ? cudaLaunchKernelEx(cfg, kea::glu_depthwise_quant_kernel<KW, 4>, a)
                       : cudaLaunchKernelEx(cfg, kea::glu_depthwise_quant_kernel<KW, 8>, a);
}

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
        case KEA_ERR_SCRATCH_LIMIT:
            return "the shape's split-K partial sums need more scratch than the no-allocation entry point's 16 MiB";
        default: return "unknown status";
    }
}

size_t kea_lowbit_panel_bytes(int32_t wbits, int32_t n, int32_t k) {
    if ((wbits != 1 && wbits != 2) || n < 1 || k < 1) return 0;
    return (size_t)ceil_div(n, kea::kPanelN) * (size_t)ceil_div(k, kea::kBK) * (size_t)wbits * kea::kPanelSubBytes;
}

size_t kea_lowbit_workspace_bytes(int32_t m, int32_t n, int32_t k, int32_t wbits, int32_t parts) {
    if (m < 1 || n < 1 || k < 1 || (wbits != 1 && wbits != 2) || parts < 1 || parts > 3) return 0;
    int sms = kSmsB200;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0) sms = v;
    }
    cudaGetLastError();   // no device here (a CPU host): size for a B200
    const KeaGemmConfig c = choose(m, n, k, wbits, parts, sms);
    return c.kernel == 1 ? pair_workspace_bytes(m, n, k, parts, sms) : 0u;
}

int kea_lowbit_gemm_noalloc(const KeaGemmDesc *d, void *stream) {
    const int v = validate_gemm(d);
    if (v != KEA_OK || d->m == 0) return v;
    int dev = 0;
    const int st = device_setup(&dev, stream);
    if (st != KEA_OK) return st;
    if (routed_scratch_bytes(d, g_devices[dev].sms) > (size_t)KEA_NOALLOC_SCRATCH_BYTES) return KEA_ERR_SCRATCH_LIMIT;
    KeaGemmDesc g = *d;
    g.workspace = g_devices[dev].noalloc_scratch;
    g.workspace_bytes = (int64_t)KEA_NOALLOC_SCRATCH_BYTES;
    return kea_lowbit_gemm(&g, stream);
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
    const int st = device_setup(&dev, stream);
    if (st != KEA_OK) return st;
    const int row_bytes = ceil_div((long long)k * wbits, 8);
    const int kb = ceil_div(k, kea::kBK);
    const long long rows = (long long)ceil_div(n, kea::kPanelN) * kb * wbits * kea::kPanelN;
    const unsigned blocks = (unsigned)((rows + 255) / 256);
    kea::prepare_panels_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(codes, row_bytes, wbits, n, k, kb, rows,
                                                                          panels, error_word);
    return cudaGetLastError() == cudaSuccess ? KEA_OK : KEA_ERR_CUDA;
}

int kea_lowbit_rel_attention(const KeaAttentionDesc *d, void *stream) {
    if (!d || !d->qkv || !d->pos || !d->bias_u || !d->bias_v || !d->ctx || d->b < 0 || d->t < 0 || d->h < 1 ||
        (d->flags & ~KEA_CONV_PDL))
        return KEA_ERR_INVALID_VALUE;
    if (d->dk != 32 && d->dk != 64 && d->dk != 128) return KEA_ERR_UNSUPPORTED;
    if (!aligned16(d->qkv) || !aligned16(d->pos) || !aligned16(d->bias_u) || !aligned16(d->bias_v) ||
        !aligned16(d->ctx))
        return KEA_ERR_ALIGNMENT;
    if (d->b == 0 || d->t == 0) return KEA_OK;
    if (d->b > 65535 || d->h > 65535) return KEA_ERR_UNSUPPORTED;
    int dev = 0;
    const int st = device_setup(&dev, stream);
    if (st != KEA_OK) return st;
    kea::RelAttnArgs a{};
    a.qkv = d->qkv;
    a.pos = d->pos;
    a.bias_u = d->bias_u;
    a.bias_v = d->bias_v;
    a.lengths = d->lengths;
    a.ctx = d->ctx;
    a.B = d->b;
    a.T = d->t;
    a.H = d->h;
    a.scale = d->scale;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(d->t, kea::kAttnQ), (unsigned)d->h, (unsigned)d->b);
    cfg.blockDim = dim3(kea::kAttnThreads, 1, 1);
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    if (d->flags & KEA_CONV_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 1;
    }
    const int sms = g_devices[dev].sms;
    const cudaError_t e = d->dk == 128 ? launch_rel_attention<128>(&cfg, a, sms)
                          : d->dk == 64 ? launch_rel_attention<64>(&cfg, a, sms) : launch_rel_attention<32>(&cfg, a, sms);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return KEA_ERR_CUDA;
    }
    return KEA_OK;
}

int kea_lowbit_glu_depthwise(const KeaConvDesc *d, void *stream) {
    if (!d || !d->h || (!d->y && !d->q) || !d->weight || d->b < 0 || d->t < 0 || d->c < 1 || d->kw < 1 ||
        d->kw % 2 == 0 || d->kw > kea::kConvMaxKw || (d->flags & ~(KEA_CONV_PDL | KEA_CONV_QUANT_SILU)))
        return KEA_ERR_INVALID_VALUE;
    const bool quant = d->q != nullptr;
    if (quant) {
        if (!d->qs || d->parts < 1 || d->parts > 3 || d->ldq < d->c) return KEA_ERR_INVALID_VALUE;
        if ((reinterpret_cast<uintptr_t>(d->q) & 3u) || d->ldq % 4 || (d->parts > 1 && d->q_part_stride % 4) ||
            (reinterpret_cast<uintptr_t>(d->h) & 15u) || (d->y && (reinterpret_cast<uintptr_t>(d->y) & 15u)))
            return KEA_ERR_ALIGNMENT;
        if (d->c % 4 || d->c > kea::kConvQMaxC || d->kw != 9) return KEA_ERR_UNSUPPORTED;   // the built fused form
    } else if (d->flags & KEA_CONV_QUANT_SILU) {
        return KEA_ERR_INVALID_VALUE;
    }
    if (d->kw != 9 && d->kw != 3 && d->kw != 31) return KEA_ERR_UNSUPPORTED;   // the built widths
    if (d->b == 0 || d->t == 0) return KEA_OK;
    if (d->b > 65535) return KEA_ERR_UNSUPPORTED;
    int dev = 0;
    const int st = device_setup(&dev, stream);
    if (st != KEA_OK) return st;
    kea::ConvArgs a{};
    a.h = d->h;
    a.y = d->y;
    a.w = d->weight;
    a.bias = d->bias;
    a.lengths = d->lengths;
    a.B = d->b;
    a.T = d->t;
    a.C = d->c;
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = {};
    if (quant) {
        kea::ConvQuantArgs qa{};
        qa.c = a;
        qa.q = d->q;
        qa.q_stride = d->q_part_stride;
        qa.ldq = d->ldq;
        qa.qs = d->qs;
        qa.qs_stride = d->qs_part_stride;
        qa.parts = d->parts;
        qa.silu = (d->flags & KEA_CONV_QUANT_SILU) ? 1 : 0;
        // 4 frames a CTA while that keeps the grid within a few waves (one clip: 32 CTAs), else 8 (fewer halo
        // re-reads for large batches)
        const int frames = (long long)d->b * ceil_div(d->t, 4) <= 4LL * g_devices[dev].sms ? 4 : 8;
        cfg.gridDim = dim3((unsigned)ceil_div(d->t, frames), (unsigned)d->b, 1);
        cfg.blockDim = dim3(kea::kConvQThreads, 1, 1);
        cfg.stream = (cudaStream_t)stream;
        cfg.attrs = attr;
        if (d->flags & KEA_CONV_PDL) {
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.numAttrs = 1;
        }
        const cudaError_t e = launch_glu_dw_quant<9>(&cfg, qa, frames);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return KEA_ERR_CUDA;
        }
        return KEA_OK;
    }
    cfg.gridDim = dim3((unsigned)ceil_div(d->c, kea::kConvThreads), (unsigned)ceil_div(d->t, kea::kConvChunk),
                       (unsigned)d->b);
    cfg.blockDim = dim3(kea::kConvThreads, 1, 1);
    cfg.stream = (cudaStream_t)stream;
    cfg.attrs = attr;
    if (d->flags & KEA_CONV_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs = 1;
    }
    const cudaError_t e = d->kw == 9 ? launch_glu_dw<9>(&cfg, a) : d->kw == 3 ? launch_glu_dw<3>(&cfg, a)
                                                                             : launch_glu_dw<31>(&cfg, a);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return KEA_ERR_CUDA;
    }
    return KEA_OK;
}

static bool quant_unit_rows(const KeaQuantizeDesc *d) {
    return d->xk == 1 && d->k % 4 == 0 && (reinterpret_cast<uintptr_t>(d->x) & 15u) == 0 && d->xt % 4 == 0 &&
           (d->t == 1 || d->xb % 4 == 0) && d->k <= 32 * kea::kQuantThreads &&
           (!d->norm_weight || (reinterpret_cast<uintptr_t>(d->norm_weight) & 15u) == 0) &&
           (!d->norm_bias || (reinterpret_cast<uintptr_t>(d->norm_bias) & 15u) == 0);
}

// Argument checks of the quantizer (KEA_OK: launchable).
static int validate_quantize(const KeaQuantizeDesc *d) {
    if (!d || !d->x || !d->q || !d->qs || d->m < 0 || d->k < 1 || d->parts < 1 || d->parts > 3 || d->t < 1 ||
        d->ldq < d->k)
        return KEA_ERR_INVALID_VALUE;
    if (d->flags & ~(KEA_QUANT_INPUT_SILU | KEA_QUANT_PDL | KEA_QUANT_NARROW_ROWS)) return KEA_ERR_INVALID_VALUE;
    if ((long long)d->k * 4 > 64 * 1024) return KEA_ERR_UNSUPPORTED;
    // codes are written as 32-bit words
    if ((reinterpret_cast<uintptr_t>(d->q) & 3u) || d->ldq % 4 || (d->parts > 1 && d->q_part_stride % 4))
        return KEA_ERR_ALIGNMENT;
    if (d->pre_norm_weight) {   // the pre-norm keeps rows in registers: unit-stride, aligned rows only
        const bool aligned = d->normed && (reinterpret_cast<uintptr_t>(d->normed) & 15u) == 0 && d->ld_normed % 4 == 0 &&
                             d->ld_normed >= d->k && (reinterpret_cast<uintptr_t>(d->pre_norm_weight) & 15u) == 0 &&
                             (!d->pre_norm_bias || (reinterpret_cast<uintptr_t>(d->pre_norm_bias) & 15u) == 0);
        if (!aligned) return d->normed ? KEA_ERR_ALIGNMENT : KEA_ERR_INVALID_VALUE;
        if (!quant_unit_rows(d)) return KEA_ERR_UNSUPPORTED;
    }
    return KEA_OK;
}

int kea_lowbit_quantize(const KeaQuantizeDesc *d, void *stream) {
    const int vq = validate_quantize(d);
    if (vq != KEA_OK) return vq;
    if ((long long)d->k * 4 > 64 * 1024) return KEA_ERR_UNSUPPORTED;
    const bool unit_rows = quant_unit_rows(d);
    if (d->m == 0) return KEA_OK;
    int dev = 0;
    const int st = device_setup(&dev, stream);
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
    a.flags = d->flags & KEA_QUANT_INPUT_SILU;
    a.pnw = d->pre_norm_weight;
    a.pnb = d->pre_norm_bias;
    a.peps = d->pre_eps;
    a.normed = d->normed;
    a.ldn = d->ld_normed;
    // Threads per row: enough CTAs to give every SM two (few rows: up to 256 threads on a row, for latency), as few
    // as one warp per row when rows are many.
    int tpr = 32;
    while (tpr < kea::kQuantThreads && (long long)ceil_div(d->m, kea::kQuantThreads / tpr) < 2LL * g_devices[dev].sms) tpr *= 2;
    cudaLaunchAttribute attr[1];
    if (unit_rows) {
        if (d->flags & KEA_QUANT_NARROW_ROWS) tpr = 32;
        // registers: at most 32 values a thread
        while (tpr < kea::kQuantThreads && d->k > 32 * tpr) tpr *= 2;
        const int vpt = round_up(ceil_div(d->k, tpr), 4);
        const dim3 grid((unsigned)ceil_div(d->m, kea::kQuantThreads / tpr));
        cudaLaunchConfig_t cfg = launch_config(grid, 0, stream, attr, d->flags & KEA_QUANT_PDL);
        cudaError_t e;
        if (vpt <= 4) e = cudaLaunchKernelEx(&cfg, kea::quantize_regs_kernel<4>, a, tpr);
        else if (vpt <= 8) e = cudaLaunchKernelEx(&cfg, kea::quantize_regs_kernel<8>, a, tpr);
        else if (vpt <= 16) e = cudaLaunchKernelEx(&cfg, kea::quantize_regs_kernel<16>, a, tpr);
        else e = cudaLaunchKernelEx(&cfg, kea::quantize_regs_kernel<32>, a, tpr);
        if (e != cudaSuccess) cudaGetLastError();
        return e == cudaSuccess ? KEA_OK : KEA_ERR_CUDA;
    }
    // shared-memory staging for other layouts; the CTA's rows must fit 64 KB
    while (tpr < kea::kQuantThreads && (kea::kQuantThreads / tpr) * d->k * (int)sizeof(float) > 64 * 1024) tpr *= 2;
    const int rows = kea::kQuantThreads / tpr;
    cudaLaunchConfig_t cfg = launch_config(dim3((unsigned)ceil_div(d->m, rows)), (size_t)rows * d->k * sizeof(float),
                                           stream, attr, d->flags & KEA_QUANT_PDL);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kea::quantize_kernel, a, tpr);
    if (e != cudaSuccess) cudaGetLastError();
    return e == cudaSuccess ? KEA_OK : KEA_ERR_CUDA;
}

}  // extern "C"

// The fused prologue quantizer of the per-tile kernel: the quantizer descriptor's input rows and options, and the
// caller's scratch for the clusters' quantized blocks.
struct FusedQuant {
    const KeaQuantizeDesc *q;
    void *scratch;
    size_t scratch_bytes;
    bool dry_run;                 // decide only: KEA_OK if the fused form applies, nothing launched
};
constexpr int kNotFused = 1000;   // launch_tile's answer when the fused form does not apply (nothing launched)

size_t fused_scratch_bytes(int clusters, int k) { return (size_t)clusters * kea::kBM * ((size_t)k + 4); }

// Clusters of kFqCluster CTAs of the per-tile kernel (wbits, one part) with `smem` bytes of dynamic shared memory
// that fit on the device at once (one wave), looked up once per (device, wbits, size) and cached.
int fused_max_clusters(int dev, int wbits, int smem) {
    struct Entry { int dev, wbits, smem, clusters; };
    static Entry cache[32];
    static int used = 0;
    std::lock_guard<std::mutex> lock(g_mutex);
    for (int i = 0; i < used; ++i)
        if (cache[i].dev == dev && cache[i].wbits == wbits && cache[i].smem == smem) return cache[i].clusters;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kea::kFqCluster, 1, 1);
    cfg.blockDim = dim3(kea::kThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kea::kFqCluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    const void *fn = wbits == 1 ? (const void *)kea::lowbit_gemm_kernel<1, 1> : (const void *)kea::lowbit_gemm_kernel<2, 1>;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    if (used < 32) cache[used++] = Entry{dev, wbits, smem, n};
    return n;
}

// The fused form stages the LayerNorms' parameters (4 K floats) in the activation region, empty until the
// quantized rows are loaded there, so it needs no more shared memory than the plain launch.
constexpr uint32_t kFqParamOffset = 0;

// The per-tile kernel's launch for the table's (or the caller's forced) tiles; with `fq`, only the fused form (one
// launch quantizing and multiplying) or kNotFused.
int launch_tile(const KeaGemmDesc *d, KeaGemmConfig c, int dev, void *stream, const FusedQuant *fq) {
    const bool forced = d->tile_m || d->tile_n || d->splits || d->stages;
    if (c.kernel) c = choose_tile(d->m, d->n, d->k, d->wbits, d->parts, g_devices[dev].sms);
    // the channel tile widened to 64 where the fused form's clusters would not all fit on the device at once (N 4096
    // at 32 channels: 16 clusters of 8 against 15 that fit at one CTA per SM)
    if (fq && !forced && c.tile_n == 32 && d->parts == 1 && c.splits == 1 &&
        ceil_div(d->n, 32) / kea::kFqCluster > fused_max_clusters(dev, d->wbits, c.smem_bytes)) {
        c.tile_n = 64;
        c.stages = std::max(1, std::min(c.stages, max_stages(c.tile_m, 64, 1, d->wbits)));
        c.smem_bytes = dyn_smem_bytes(c.tile_m, 64, 1, d->wbits, c.splits, c.stages);
    }
    // Stacked parts (one 128-row tile holds every part's tokens): pe is the parts the tile's footprint counts.
    // forced tiles may stack whenever the shape allows; the table stacks where it chose to
    int pe = (forced ? stackable(d->m, d->parts, d->k) : use_stack(d->m, d->n, d->k, d->parts, g_devices[dev].sms))
                 ? 1 : d->parts;
    if (forced) {
        if (d->tile_m) c.tile_m = d->tile_m;
        if (d->tile_n) c.tile_n = d->tile_n;
        if (d->splits) c.splits = d->splits;
        if (c.tile_m != kea::kBM) pe = d->parts;
        if (d->stages) {
            c.stages = d->stages;
        } else {
            const int per = ceil_div(ceil_div(d->k, kea::kBK), std::max(1, c.splits));
            c.stages = std::max(1, std::min(per, max_stages(c.tile_m, c.tile_n, pe, d->wbits)));
        }
        c.smem_bytes = dyn_smem_bytes(c.tile_m, c.tile_n, pe, d->wbits, c.splits, c.stages);
    }
    // the single-tile stacked epilogue stages every TMEM row (TN + 4 words) in the stage area
    const bool stack = pe == 1 && d->parts > 1 && c.tile_m == kea::kBM &&
                       (c.splits > 1 || kea::kBM * (c.tile_n + 4) * 4 <= c.stages * stage_bytes(c.tile_m, c.tile_n, 1, d->wbits));
    if (!stack && pe == 1 && d->parts > 1) {   // footprint sized for stacking that cannot be used: size for the parts
        pe = d->parts;
        if (!forced) c = choose_tile(d->m, d->n, d->k, d->wbits, d->parts, g_devices[dev].sms, false);
        else c.smem_bytes = dyn_smem_bytes(c.tile_m, c.tile_n, pe, d->wbits, c.splits, c.stages);
    }
    const int cs = check_config(c, d->n, d->k, pe, d->wbits);
    if (cs != KEA_OK) return cs;

    // Activations. When K is a multiple of 128: a 4-D view (k within a 128-block, row, k-block, part) whose boxes are
    // 128 k x (128 * token blocks) rows x kbox k-blocks x 1 part, so one TMA instruction fills a part's token blocks
    // (and, in one-shot mode, several k-blocks). Otherwise a 3-D view (k, row, part) with 128 x 128 boxes, whose
    // columns >= k read as zero. Both use the 128-byte swizzle of the tcgen05 K-major layout; rows >= m read as 0.
    const int tmb = c.tile_m / kea::kBM;
    const int kb_total = ceil_div(d->k, kea::kBK);
    const int nkb_max = ceil_div(kb_total, c.splits);
    const bool q4d = d->k % kea::kBK == 0;
    const int R = std::min(c.tile_n, kea::kPanelN);
    // One-shot: the CTA's whole K range fits in the stages and arrives in two TMA boxes (one token block, one
    // part, narrow channel tile so the panel box is at most 256 bytes wide).
    const bool oneshot = q4d && tmb * pe == 1 && c.tile_n <= 64 && nkb_max <= c.stages && nkb_max <= 8;
    // two chunks when they fit the stages: the second lands while the first is expanded and multiplied
    const int chunks = oneshot && nkb_max >= 4 && 2 * ceil_div(nkb_max, 2) <= c.stages ? 2 : 1;
    const int kbox = oneshot ? ceil_div(nkb_max, chunks) : 1;
    // The fused quantizer: one token tile of one part, the whole K (<= 1024, whole 128-blocks) in one shot, channel
    // tiles in whole clusters of kFqCluster, unit-stride 16-byte-aligned input rows.
    int fq_clusters = 0;
    uint32_t fq_off = 0;
    if (fq) {
        const KeaQuantizeDesc *x = fq->q;
        const int ctas_n = ceil_div(d->n, c.tile_n);
        const bool shape_ok = oneshot && !stack && pe == 1 && d->parts == 1 && c.splits == 1 && tmb == 1 &&
                              d->m <= kea::kBM && d->k % kea::kBK == 0 && d->k <= kea::kRowChunks * 128 &&
                              ctas_n % kea::kFqCluster == 0;
        bool rows_ok = x->xk == 1 && aligned16(x->x) && x->xt % 4 == 0 && (x->t == 1 || x->xb % 4 == 0) &&
                       (!x->pre_norm_weight || (x->normed && aligned16(x->normed) && x->ld_normed % 4 == 0));
        if (rows_ok && x->pre_norm_weight) {
            // cluster 0 writes the pre-norm output while other clusters still read the input rows: not in place
            const long long last = (long long)(d->m - 1) / x->t * x->xb + (long long)(x->t - 1) * x->xt + d->k;
            const uintptr_t x0 = reinterpret_cast<uintptr_t>(x->x), x1 = x0 + (uintptr_t)last * 4;
            const uintptr_t n0 = reinterpret_cast<uintptr_t>(x->normed);
            const uintptr_t n1 = n0 + ((uintptr_t)(d->m - 1) * x->ld_normed + d->k) * 4;
            if (x0 < n1 && n0 < x1) rows_ok = false;
        }
        fq_clusters = ctas_n / kea::kFqCluster;
        fq_off = kFqParamOffset;
        const bool room = c.stages * a_stage_bytes(c.tile_m, 1) >= 4 * d->k * 4;   // the activation region
        if (!shape_ok || !rows_ok || !room || !fq->scratch || !aligned16(fq->scratch) ||
            fq->scratch_bytes < fused_scratch_bytes(fq_clusters, d->k))
            return kNotFused;
        if (fq->dry_run) return KEA_OK;
    }
    CUtensorMap qmap;
    const long long pstride = d->parts > 1 ? d->q_part_stride : (long long)d->m * d->ldq;
    // Rows past m only feed accumulator rows that are never stored, so a single token tile loads just the rows
    // that exist (rounded up to the 8-row swizzle atom) instead of zero-filling the rest.
    const int box_rows4 = stack ? stack_rows(d->m, d->parts, d->k) : std::min(kea::kBM * tmb, round_up(d->m, 8));
    const int box_rows3 = std::min(kea::kBM, round_up(d->m, 8));
    uint32_t act_tx;
    if (q4d && stack) {
        // (k in block, row, part, k-block): one box = box_rows4 rows of every part for kbox k-blocks, landing as
        // [k-block][part][row][128 bytes], i.e. the parts stacked along the tile's rows
        act_tx = (uint32_t)(d->parts * box_rows4 * kea::kBK);
        const cuuint64_t dims[4] = {(cuuint64_t)kea::kBK, (cuuint64_t)d->m, (cuuint64_t)d->parts, (cuuint64_t)kb_total};
        const cuuint64_t strides[3] = {(cuuint64_t)d->ldq, (cuuint64_t)std::max<long long>(pstride, 16), (cuuint64_t)kea::kBK};
        const cuuint32_t box[4] = {(cuuint32_t)kea::kBK, (cuuint32_t)box_rows4, (cuuint32_t)d->parts, (cuuint32_t)kbox};
        const cuuint32_t estr[4] = {1, 1, 1, 1};
        if (g_encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<int8_t *>(d->q), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return KEA_ERR_CUDA;
    } else if (q4d) {
        act_tx = (uint32_t)(d->parts * box_rows4 * kea::kBK);
        // fused: the clusters' scratch blocks [cluster][128 rows][K] stand in for q
        const cuuint64_t rows = fq ? (cuuint64_t)fq_clusters * kea::kBM : (cuuint64_t)d->m;
        const cuuint64_t ld = fq ? (cuuint64_t)d->k : (cuuint64_t)d->ldq;
        void *src = fq ? fq->scratch : const_cast<int8_t *>(d->q);
        const long long ps = fq ? (long long)rows * d->k : pstride;
        const cuuint64_t dims[4] = {(cuuint64_t)kea::kBK, rows, (cuuint64_t)kb_total, (cuuint64_t)d->parts};
        const cuuint64_t strides[3] = {ld, (cuuint64_t)kea::kBK, (cuuint64_t)std::max<long long>(ps, 16)};
        const cuuint32_t box[4] = {(cuuint32_t)kea::kBK, (cuuint32_t)box_rows4, (cuuint32_t)kbox, 1};
        const cuuint32_t estr[4] = {1, 1, 1, 1};
        if (g_encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, src, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return KEA_ERR_CUDA;
    } else {
        act_tx = (uint32_t)(tmb * d->parts * box_rows3 * kea::kBK);
        const cuuint64_t dims[3] = {(cuuint64_t)d->k, (cuuint64_t)d->m, (cuuint64_t)d->parts};
        const cuuint64_t strides[2] = {(cuuint64_t)d->ldq, (cuuint64_t)std::max<long long>(pstride, 16)};
        const cuuint32_t box[3] = {(cuuint32_t)kea::kBK, (cuuint32_t)box_rows3, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        if (g_encode(&qmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<int8_t *>(d->q), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return KEA_ERR_CUDA;
    }
    // Panels in one-shot mode: a 2-D view (byte within one 512-byte word plane, plane), plane index
    // ((tile * kb_total + k-block) * wbits + sub-block) * 4 + word; a box takes this CTA's R rows of kbox * wbits * 4
    // consecutive planes.
    CUtensorMap wmap;
    std::memset(&wmap, 0, sizeof(wmap));
    if (oneshot) {
        const long long planes = (long long)ceil_div(d->n, kea::kPanelN) * kb_total * d->wbits * 4;
        const cuuint64_t dims[2] = {(cuuint64_t)(kea::kPanelN * 4), (cuuint64_t)planes};
        const cuuint64_t strides[1] = {(cuuint64_t)(kea::kPanelN * 4)};
        const cuuint32_t box[2] = {(cuuint32_t)(R * 4), (cuuint32_t)(kbox * d->wbits * 4)};
        const cuuint32_t estr[2] = {1, 1};
        if (g_encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(d->panels), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return KEA_ERR_CUDA;
    }

    // Output: TMA stores of 32-row x tile_n / 4-column boxes when the row stride allows (16-byte multiple) and a
    // warp's staged row is 64 or 128 bytes (the swizzle span of the shared-memory staging).
    CUtensorMap ymap;
    std::memset(&ymap, 0, sizeof(ymap));
    const int out_esize = d->y_dtype == KEA_OUT_F16 ? 2 : 4;
    const int warp_row_bytes = (c.tile_n / 4) * out_esize;
    const int staging_bytes = (c.tile_m / kea::kBM) * kea::kEpiWarps * 32 * warp_row_bytes;   // reuses the stages
    // (a residual is added by the direct-store epilogue, which reads it next to the value it finishes)
    bool tma_store = c.splits == 1 && !d->residual && aligned16(d->y) && (d->ldy * out_esize) % 16 == 0 &&
                     (warp_row_bytes == 64 || warp_row_bytes == 128) &&
                     staging_bytes <= c.stages * stage_bytes(c.tile_m, c.tile_n, pe, d->wbits);
    if (tma_store) {
        const cuuint64_t ydims[2] = {(cuuint64_t)d->n, (cuuint64_t)d->m};
        const cuuint64_t ystrides[1] = {(cuuint64_t)(d->ldy * out_esize)};
        const cuuint32_t ybox[2] = {(cuuint32_t)(c.tile_n / 4), 32};
        const cuuint32_t yestr[2] = {1, 1};
        if (g_encode(&ymap, out_esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, d->y,
                     ydims, ystrides, ybox, yestr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     warp_row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            tma_store = false;
    }

    GemmArgs a{};
    a.tma_store = tma_store ? 1 : 0;
    a.store_swizzle = warp_row_bytes;
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
    a.tile_n = c.tile_n;
    a.tm_blocks = c.tile_m / kea::kBM;
    a.splits = c.splits;
    a.stages = c.stages;
    a.kb_total = ceil_div(d->k, kea::kBK);
    a.flags = d->flags & (KEA_FLAG_SILU | KEA_FLAG_ORDER1);
    a.res = d->residual;
    a.ld_res = d->ld_residual;
    a.res_scale = d->residual_scale;
    a.pdl = (d->flags & KEA_FLAG_PDL) ? 1 : 0;
    a.tmem_cols = tmem_columns(c.tile_m, c.tile_n, pe);
    a.a_stage = (uint32_t)a_stage_bytes(c.tile_m, pe);
    a.b_stage = (uint32_t)b_stage_bytes(c.tile_n);
    a.pk_stage = (uint32_t)pk_stage_bytes(c.tile_n, d->wbits);
    a.b_region = (uint32_t)c.stages * a.a_stage;
    a.pk_region = a.b_region + (uint32_t)c.stages * a.b_stage;
    a.q4d = q4d ? 1 : 0;
    a.oneshot = oneshot ? 1 : 0;
    a.chunks = chunks;
    a.kbox = kbox;
    a.act_tx = act_tx;
    a.nacc = accumulators(c.tile_m, c.tile_n, pe);
    a.a_stride = oneshot ? (uint32_t)((stack ? d->parts : 1) * box_rows4 * kea::kBK) : a.a_stage;
    a.recv_aliases_stages = exchange_aliases(c.tile_m, c.tile_n, pe, d->wbits, c.splits, c.stages) ? 1 : 0;
    a.recv_off = a.recv_aliases_stages ? 0u : (uint32_t)(c.stages * stage_bytes(c.tile_m, c.tile_n, pe, d->wbits));
    a.stack = stack ? 1 : 0;
    a.mp = box_rows4;
    a.res = d->residual;
    a.ld_res = d->ld_residual;
    a.res_scale = d->residual_scale;
    const int esize = d->y_dtype == KEA_OUT_F16 ? 2 : 4;
    a.vec_y = aligned16(d->y) && ((d->ldy * esize) % 16 == 0);
    a.vec_acc = d->acc && aligned16(d->acc) && ((d->ld_acc * 4) % 16 == 0) && ((d->acc_part_stride * 4) % 16 == 0);
    a.err = d->error_word;
    if (fq) {
        const KeaQuantizeDesc *x = fq->q;
        a.fq = 1;
        a.fq_x = x->x;
        a.fq_xb = x->xb;
        a.fq_xt = x->xt;
        a.fq_t = x->t;
        a.fq_silu = (x->flags & KEA_QUANT_INPUT_SILU) ? 1 : 0;
        a.fq_nw = x->norm_weight;
        a.fq_nb = x->norm_bias;
        a.fq_eps = x->eps;
        a.fq_pnw = x->pre_norm_weight;
        a.fq_pnb = x->pre_norm_bias;
        a.fq_peps = x->pre_eps;
        a.fq_off = fq_off;
        a.fq_scr = static_cast<int8_t *>(fq->scratch);
        a.fq_qs_scr = reinterpret_cast<float *>(static_cast<int8_t *>(fq->scratch) +
                                                (size_t)fq_clusters * kea::kBM * d->k);
        a.fq_q = const_cast<int8_t *>(d->q);
        a.fq_qs = const_cast<float *>(d->qs);
        a.fq_ldq = d->ldq;
        a.fq_normed = x->pre_norm_weight ? x->normed : nullptr;
        a.fq_ldn = x->ld_normed;
    }

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)ceil_div(d->n, c.tile_n),
                       (unsigned)(stack ? ceil_div(d->m, box_rows4) : ceil_div(d->m, c.tile_m)), (unsigned)c.splits);
    cfg.blockDim = dim3(kea::kThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)c.smem_bytes;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attrs[2];
    unsigned na = 0;
    if (c.splits > 1 || fq) {
        attrs[na].id = cudaLaunchAttributeClusterDimension;
        attrs[na].val.clusterDim.x = fq ? (unsigned)kea::kFqCluster : 1u;
        attrs[na].val.clusterDim.y = 1;
        attrs[na].val.clusterDim.z = fq ? 1u : (unsigned)c.splits;
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
        case 5: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<1, 1>, qmap, ymap, wmap, a); break;
        case 6: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<1, 2>, qmap, ymap, wmap, a); break;
        case 7: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<1, 3>, qmap, ymap, wmap, a); break;
        case 9: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<2, 1>, qmap, ymap, wmap, a); break;
        case 10: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<2, 2>, qmap, ymap, wmap, a); break;
        default: e = cudaLaunchKernelEx(&cfg, kea::lowbit_gemm_kernel<2, 3>, qmap, ymap, wmap, a); break;
    }
    if (e != cudaSuccess) {
        cudaGetLastError();
        return KEA_ERR_CUDA;
    }
    return KEA_OK;
}

extern "C" {

int kea_lowbit_gemm(const KeaGemmDesc *d, void *stream) {
    const int v = validate_gemm(d);
    if (v != KEA_OK || d->m == 0) return v;
    int dev = 0;
    const int st = device_setup(&dev, stream);
    if (st != KEA_OK) return st;
    Route route;
    KeaGemmConfig c{};
    SwapPlan sp;
    RegPlan rp;
    const int rs = route_gemm(d, g_devices[dev].sms, &route, &c, &sp, &rp);
    if (rs != KEA_OK) return rs;
    if (route == kRouteGemv) return launch_gemv(d, c, stream);
    if (route == kRouteReg) return launch_reg(d, rp, stream);
    if (route == kRouteSwap) return launch_swap(d, sp, stream);
    if (route == kRoutePair) return launch_pair(d, c, g_devices[dev].sms, stream);
    return launch_tile(d, c, dev, stream, nullptr);
}

size_t kea_lowbit_project_scratch_bytes(int32_t m, int32_t n, int32_t k, int32_t wbits, int32_t parts) {
    (void)wbits;
    if (m < 1 || m > kea::kBM || n < 1 || parts != 1 || k < 1 || k % kea::kBK || k > kea::kRowChunks * 128) return 0;
    // at most one cluster per kFqCluster channel tiles of the narrowest (32-channel) tile
    return fused_scratch_bytes(ceil_div(ceil_div(n, 32), kea::kFqCluster), k);
}

// The route kea_lowbit_project takes (fused 1: one fused kernel; 0: quantizer then GEMM) after its argument checks,
// with the per-tile configuration and device the fused launch uses.
static int project_route(const KeaProjectDesc *p, void *stream, int *fused, KeaGemmConfig *cfg, int *device) {
    *fused = 0;
    if (!p) return KEA_ERR_INVALID_VALUE;
    const KeaGemmDesc *d = &p->gemm;
    const KeaQuantizeDesc *x = &p->quant;
    const int v = validate_gemm(d);
    if (v != KEA_OK) return v;
    const int vq = validate_quantize(x);
    if (vq != KEA_OK) return vq;
    if (p->flags & ~KEA_PROJECT_FUSE) return KEA_ERR_INVALID_VALUE;
    // the quantizer's output is the GEMM's input
    if (x->m != d->m || x->k != d->k || x->parts != d->parts || x->q != d->q || x->ldq != d->ldq || x->qs != d->qs ||
        (d->parts > 1 && (x->q_part_stride != d->q_part_stride || x->qs_part_stride != d->qs_part_stride)))
        return KEA_ERR_INVALID_VALUE;
    if (d->m == 0) return KEA_OK;
    int dev = 0;
    const int st = device_setup(&dev, stream);
    if (st != KEA_OK) return st;
    Route route;
    KeaGemmConfig c{};
    SwapPlan sp;
    RegPlan rp;
    // the fused form lives in the per-tile tcgen05 kernel: a caller asking for it routes as if the register kernel
    // were off (unless it forces that kernel)
    KeaGemmDesc g = *d;
    if ((p->flags & KEA_PROJECT_FUSE) && !(g.flags & KEA_FLAG_FORCE_REG)) g.flags |= KEA_FLAG_NO_REG;
    const int rs = route_gemm(&g, g_devices[dev].sms, &route, &c, &sp, &rp);
    if (rs != KEA_OK) return rs;
    if ((p->flags & KEA_PROJECT_FUSE) && route == kRouteTile && quant_unit_rows(x)) {
        const FusedQuant fq{x, p->scratch, p->scratch_bytes, true};
        *fused = launch_tile(d, c, dev, stream, &fq) == KEA_OK ? 1 : 0;
    }
    *cfg = c;
    *device = dev;
    return KEA_OK;
}

int kea_lowbit_project_fuses(const KeaProjectDesc *p) {
    int fused = 0, dev = 0;
    KeaGemmConfig c{};
    const int st = project_route(p, nullptr, &fused, &c, &dev);
    return st != KEA_OK ? -st : fused;
}

int kea_lowbit_project(const KeaProjectDesc *p, void *stream) {
    int fused = 0, dev = 0;
    KeaGemmConfig c{};
    const int st = project_route(p, stream, &fused, &c, &dev);
    if (st != KEA_OK || p->gemm.m == 0) return st;
    if (fused) {
        const FusedQuant fq{&p->quant, p->scratch, p->scratch_bytes, false};
        const int r = launch_tile(&p->gemm, c, dev, stream, &fq);
        if (r != kNotFused) return r;
    }
    const int q = kea_lowbit_quantize(&p->quant, stream);
    if (q != KEA_OK) return q;
    return kea_lowbit_gemm(&p->gemm, stream);
}


int kea_lowbit_read_error(uint32_t *out) {
    if (!out) return KEA_ERR_INVALID_VALUE;
    int dev = 0;
    const int st = device_setup(&dev, nullptr, false);
    if (st != KEA_OK) return st;
    uint32_t v = 0;
    if (cudaMemcpyFromSymbol(&v, kea::g_device_error, sizeof(v)) != cudaSuccess) return KEA_ERR_CUDA;
    const uint32_t zero = 0;
    if (cudaMemcpyToSymbol(kea::g_device_error, &zero, sizeof(zero)) != cudaSuccess) return KEA_ERR_CUDA;
    *out = v;
    return KEA_OK;
}

}  // extern "C"
