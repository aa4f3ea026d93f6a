// C-ABI implementation of the sm_100a HGEMM library (include/hgemm_sm100.h):
// argument checks, the `auto` shape heuristic, TMA descriptor encoding and
// caching, and kernel launches on the caller's stream.
//
// Counterpart of the reference's host dispatch (csrc/dispatch.cpp:47-96) and
// of the per-backend launchers (csrc/v6_mma_async.cu:408-486 and friends),
// without torch types: the torch-facing checks live in the pybind11 module.
#include "hgemm_sm100.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstring>
#include <mutex>
#include <random>
#include <unordered_map>

#include "hgemm_kernels.cuh"

namespace {

using namespace hgemm;

static_assert(kEpiBias == HGEMM_SM100_EPI_BIAS && kEpiResidual == HGEMM_SM100_EPI_RESIDUAL &&
                  kEpiSiluMul == HGEMM_SM100_EPI_SILU_MUL,
              "kernel epilogue bits match the C ABI");
static_assert(sizeof(void*) != 8 || sizeof(HgemmSm100Args) == 152, "HgemmSm100Args layout (ctypes mirror)");

__device__ int g_status_word;  // status word used when the caller passes none

// Scratch of hgemm_sm100_run_static_scratch, for callers that cannot allocate:
// a file-scope device array that every GPU loading this library holds until
// the process exits. In host code the name is only a handle for the symbol,
// never a device address; device_info() looks its address up once per device.
static __device__ __align__(256) unsigned char g_static_scratch[HGEMM_SM100_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
constexpr int kMaxSplit = 16;
constexpr uint64_t kDefaultTimeoutNs = 2000ull * 1000ull * 1000ull;

const char* const kConfigNames[HGEMM_SM100_CFG_COUNT] = {
    "auto",
    "tc_persistent_128x256",
    "tc_persistent_128x128",
    "tc_splitk_128x128",
    "tc_swapab",
    "tc_generic_128x128",
    "tc_pair_256x256",
    "tc_splitk_128x256",
    "tc_streamk_128x256",
    "tc_streamk_swapab",
    "tc_pair_256x128",
    "tc_pair_128x256",
    "tc_pair_128x128",
    "tc_streamk_pair_256x256",
};

// ------------------------------------------------------ device properties --

struct DeviceInfo {
    int sms = 0;
    int major = 0, minor = 0;
    int* status_word = nullptr;
    uint8_t* static_scratch = nullptr;   // device address of g_static_scratch
    int max_cluster = 8;
};

DeviceInfo g_devices[kMaxDevices];
std::once_flag g_device_once[kMaxDevices];
int g_device_error[kMaxDevices];

int device_info(const DeviceInfo** out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return HGEMM_SM100_ERR_CUDA;
    std::call_once(g_device_once[dev], [dev] {
        DeviceInfo& d = g_devices[dev];
        int err = 0;
        err |= cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess;
        err |= cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess;
        err |= cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess;
        if (!err && d.major == 10 && d.minor == 0) {
            // With `dev` current: the device addresses of the library's own
            // status word and static scratch on this device.
            err |= cudaGetSymbolAddress(reinterpret_cast<void**>(&d.status_word), g_status_word) !=
                   cudaSuccess;
            err |= cudaGetSymbolAddress(reinterpret_cast<void**>(&d.static_scratch), g_static_scratch) !=
                   cudaSuccess;
            err |= d.status_word == nullptr || d.static_scratch == nullptr;
        }
        g_device_error[dev] = err ? HGEMM_SM100_ERR_CUDA
                                  : ((d.major == 10 && d.minor == 0) ? HGEMM_SM100_OK
                                                                     : HGEMM_SM100_ERR_UNSUPPORTED_DEVICE);
    });
    *out = &g_devices[dev];
    return g_device_error[dev];
}

// ------------------------------------------------------------ tensor maps --

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

struct MapKey {
    const void* base;
    uint64_t inner, outer, ld;
    uint32_t box_inner, box_outer;
    bool swizzle;
    bool operator==(const MapKey& o) const {
        return base == o.base && inner == o.inner && outer == o.outer && ld == o.ld &&
               box_inner == o.box_inner && box_outer == o.box_outer && swizzle == o.swizzle;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        size_t h = reinterpret_cast<size_t>(k.base);
        h ^= (k.inner * 0x9E3779B97F4A7C15ull) + (h << 6) + (h >> 2);
        h ^= (k.outer * 0xC2B2AE3D27D4EB4Full) + (h << 6) + (h >> 2);
        h ^= (k.ld * 0x165667B19E3779F9ull) + (h << 6) + (h >> 2);
        h ^= (static_cast<size_t>(k.box_inner) << 32 | k.box_outer) + (h << 6) + (h >> 2);
        h ^= static_cast<size_t>(k.swizzle);
        return h;
    }
};

// 2-D FP16 row-major matrix [outer x inner] with row pitch `ld` elements,
// 128-byte swizzled (or, with swizzle false, dense row-major) boxes of
// [box_outer x box_inner]; out-of-range elements read as zero. Descriptors are cached per thread (they depend only on the
// key, so a reused address with the same shape reuses a valid descriptor).
int tensor_map(CUtensorMap* out, const void* base, uint64_t inner, uint64_t outer, uint64_t ld,
               uint32_t box_inner, uint32_t box_outer, bool swizzle = true) {
    thread_local std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    const MapKey key{base, inner, outer, ld, box_inner, box_outer, swizzle};
    auto it = cache.find(key);
    if (it != cache.end()) {
        *out = it->second;
        return HGEMM_SM100_OK;
    }
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return HGEMM_SM100_ERR_TENSOR_MAP;
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap map;
    const CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                          swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return HGEMM_SM100_ERR_TENSOR_MAP;
    if (cache.size() >= 256) cache.clear();
    cache.emplace(key, map);
    *out = map;
    return HGEMM_SM100_OK;
}

// ---------------------------------------------------------------- kernels --

using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, GemmParams);

struct KernelEntry {
    const void* fn;
    uint32_t smem;
    std::atomic<uint64_t> ready{0};  // bit d: attributes set on device d
};

template <typename Cfg>
constexpr uint32_t smem_of() { return Cfg::kSmemBytes; }

int prepare_kernel(KernelEntry& k, int dev) {
    const uint64_t bit = 1ull << dev;
    if (k.ready.load(std::memory_order_acquire) & bit) return HGEMM_SM100_OK;
    if (cudaFuncSetAttribute(k.fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(k.smem)) != cudaSuccess)
        return HGEMM_SM100_ERR_LAUNCH;
    if (cudaFuncSetAttribute(k.fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
        return HGEMM_SM100_ERR_LAUNCH;
    k.ready.fetch_or(bit, std::memory_order_acq_rel);
    return HGEMM_SM100_OK;
}

#define HG_TILE(BN, SWAP, TMA, ST)                                                        \
    KernelEntry {                                                                          \
        reinterpret_cast<const void*>(&hgemm_tile_kernel<BN, SWAP, TMA, ST>),              \
            TileCfg<BN, SWAP, TMA, ST>::kSmemBytes                                         \
    }
#define HG_PAIR(BM, BN, ST)                                                                        \
    KernelEntry {                                                                                   \
        reinterpret_cast<const void*>(&hgemm_pair_kernel<BM, BN, ST>), PairCfg<BM, BN, ST>::kSmemBytes \
    }
#define HG_STREAMK(BN, SWAP, ST)                                                          \
    KernelEntry {                                                                          \
        reinterpret_cast<const void*>(&hgemm_streamk_kernel<BN, SWAP, ST>),                \
            StreamKCfg<BN, SWAP, ST>::kSmemBytes                                           \
    }
#define HG_PERSIST(BN, ST)                                                                \
    KernelEntry {                                                                          \
        reinterpret_cast<const void*>(&hgemm_persistent_kernel<BN, ST>),                   \
            PersistCfg<BN, ST>::kSmemBytes                                                 \
    }

KernelEntry g_pair_256 = HG_PAIR(256, 256, 6);
KernelEntry g_pair_128 = HG_PAIR(256, 128, 8);
KernelEntry g_pair_m128_256 = HG_PAIR(128, 256, 8);
KernelEntry g_pair_m128_128 = HG_PAIR(128, 128, 12);
KernelEntry g_pair_sk_256 = KernelEntry{reinterpret_cast<const void*>(&hgemm_pair_streamk_kernel<6>),
                                        PairCfg<256, 256, 6>::kSmemBytes};
KernelEntry g_sk_256 = HG_STREAMK(256, false, 4);
KernelEntry g_sk_swap_16 = HG_STREAMK(16, true, 10);
KernelEntry g_sk_swap_32 = HG_STREAMK(32, true, 9);
KernelEntry g_sk_swap_64 = HG_STREAMK(64, true, 8);
KernelEntry g_sk_swap_128 = HG_STREAMK(128, true, 6);
KernelEntry g_persist_256 = HG_PERSIST(256, 4);
KernelEntry g_persist_128 = HG_PERSIST(128, 6);
KernelEntry g_splitk_128 = HG_TILE(128, false, true, 6);
KernelEntry g_splitk_256 = HG_TILE(256, false, true, 4);
KernelEntry g_generic_128 = HG_TILE(128, false, false, 4);
// Swap-AB tiles (decode and small M): rings of 196-216 KB (4-12 stages by
// width), one CTA per SM, so that each SM keeps about as many weight bytes in
// flight as its loads need to stream at full rate.
KernelEntry g_swap_16 = HG_TILE(16, true, true, 12);
KernelEntry g_swap_32 = HG_TILE(32, true, true, 10);
KernelEntry g_swap_64 = HG_TILE(64, true, true, 8);
KernelEntry g_swap_128 = HG_TILE(128, true, true, 6);
KernelEntry g_swap_256 = HG_TILE(256, true, true, 4);

struct SwapChoice {
    int bnm;
    KernelEntry* k;
    int per_sm;   // CTAs that fit on one SM (1 with the rings above)
};
SwapChoice swap_of_width(int bnm) {
    switch (bnm) {
        case 16: return {16, &g_swap_16, 1};
        case 32: return {32, &g_swap_32, 1};
        case 64: return {64, &g_swap_64, 1};
        case 128: return {128, &g_swap_128, 1};
        default: return {256, &g_swap_256, 1};
    }
}

int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// K splits for a tile kernel: enough clusters to cover the SMs once, at most
// one K block per split, at most the cluster limit.
int choose_split(int64_t base_ctas, int64_t nkb, int sms, int max_split) {
    int64_t s = sms / (base_ctas > 0 ? base_ctas : 1);
    if (s < 1) s = 1;
    if (s > max_split) s = max_split;
    if (s > nkb) s = nkb;
    return static_cast<int>(s);
}

// How many clusters of `cluster` CTAs of kernel `k` fit on device `dev` at
// once (cached). Clusters must fit inside one GPC, so large clusters of
// SM-filling CTAs can fit fewer times than SMs / cluster suggests.
int max_active_clusters(KernelEntry& k, int dev, int cluster) {
    static std::mutex mu;
    static std::unordered_map<uint64_t, int> cache;
    const uint64_t key = (reinterpret_cast<uint64_t>(k.fn) << 12) ^ (static_cast<uint64_t>(dev) << 6) ^
                         static_cast<uint64_t>(cluster);
    {
        std::lock_guard<std::mutex> lock(mu);
        auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    int n = 0;
    if (prepare_kernel(k, dev) == HGEMM_SM100_OK) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(1, 1, static_cast<unsigned>(cluster));
        cfg.blockDim = dim3(kThreads, 1, 1);
        cfg.dynamicSmemBytes = k.smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 1;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = static_cast<unsigned>(cluster);
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, k.fn, &cfg) != cudaSuccess) {
            (void)cudaGetLastError();
            n = 0;
        }
    }
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = n;
    return n;
}

// Lowers `split` until all `base` clusters of the tile kernel are resident at
// once (a second wave of clusters would double the time), when possible.
int fit_split(KernelEntry& k, int dev, int64_t base, int split) {
    while (split > 1) {
        const int n = max_active_clusters(k, dev, split);
        if (n <= 0 || base <= n) break;
        --split;
    }
    return split;
}

// ------------------------------------------------- tile-kernel cost model --
//
// Device time (microseconds, constant launch / first-load / store costs
// left out) of one tile-kernel launch: `tiles` output tiles of `width`
// accumulator columns, K split `split` ways over `nkb` K blocks, `per_wave`
// CTAs resident at once, `bytes` of operands read from HBM. Constants were
// measured on B200 with back-to-back launches on inputs larger than L2:
// per-K-block time of one CTA by tile width (16: 0.15 us, 32: 0.16, 64: 0.18,
// 128: 0.22, 256: 0.34 - the MMA issue and TMA feed limits of one SM), HBM
// at 6.5 TB/s but at most 120 GB/s per streaming CTA, and the split-K
// exchange (cluster barrier and reduction; partial tiles through distributed
// shared memory up to 128 columns, through L2 above) at 1.2 us + 0.04 us per
// KB of FP32 partial tile, respectively 2 us + 0.05 us per KB.
double tile_cost(int64_t tiles, int width, int split, int64_t nkb, double bytes, int per_wave) {
    const double c = width <= 16 ? 0.15 : width <= 32 ? 0.16 : width <= 64 ? 0.18 : width <= 128 ? 0.22 : 0.34;
    const int64_t wave = per_wave > 0 ? per_wave : 1;
    const int64_t ctas = tiles * split;
    const int64_t waves = cdiv(ctas, wave);
    const double t_main = static_cast<double>(waves) * static_cast<double>(cdiv(nkb, split)) * c;
    const double streams = static_cast<double>(ctas < wave ? ctas : wave) * 0.12e6;   // bytes per us
    const double t_mem = bytes / (streams < 6.5e6 ? streams : 6.5e6);
    const double kb_partial = 128.0 * width * 4.0 / 1024.0;
    const double t_x = split <= 1 ? 0.0 : width <= 128 ? 1.2 + 0.04 * kb_partial : 2.0 + 0.05 * kb_partial;
    return (t_main > t_mem ? t_main : t_mem) + t_x;
}

// CTAs of kernel `k` resident at once in clusters of `split` (one per SM).
int wave_ctas(KernelEntry& k, int split, int sms) {
    int devid = 0;
    if (split > 1 && cudaGetDevice(&devid) == cudaSuccess) {
        const int n = max_active_clusters(k, devid, split);
        if (n > 0) return n * split;
    }
    return sms / split * split;
}

struct TilePlan {
    int32_t cfg;
    int width;     // swapped: accumulator columns (output rows) per tile; else 256
    int32_t split;
};

// K blocks of a tile configuration (TileCfg::kKB = 64 for every width); a
// K split never exceeds their number.
int64_t tile_kblocks(int32_t cfg, int width, int64_t k) {
    (void)cfg;
    (void)width;
    return cdiv(k, kBlockK);
}

// Cheapest tile-kernel plan for (m, n, k): swapped tiles of 16..256 output
// rows, and (with_wide) 128 x 256 split-K tiles; every K split up to the
// cluster limit, or only `fixed_split` when given.
TilePlan plan_tiles_uncached(int64_t m, int64_t n, int64_t k, int sms, int max_split, bool with_swap,
                             bool with_wide, int32_t fixed_split) {
    const int64_t nkb = cdiv(k, kBlockK);
    const double bytes = 2.0 * static_cast<double>(m * k + k * n);
    TilePlan best{HGEMM_SM100_CFG_SWAPAB, 128, 1};
    double best_t = -1.0;
    auto consider = [&](int32_t cfg, int width, int64_t tiles, KernelEntry& ke) {
        const int64_t blocks = tile_kblocks(cfg, width, k);
        if (fixed_split > blocks) return;   // a given split needs that many K blocks
        const int lo = fixed_split > 0 ? fixed_split : 1;
        const int hi = fixed_split > 0 ? fixed_split : (max_split < blocks ? max_split : static_cast<int>(blocks));
        for (int s = lo; s <= hi; ++s) {
            // Automatic splits: the cluster sizes the constants were measured
            // with, in one wave (waves of clusters cost far more than modelled).
            if (fixed_split <= 0 && s != 1 && s != 2 && s != 3 && s != 4 && s != 6 && s != 8 && s != 16) continue;
            const int wave = wave_ctas(ke, s, sms);
            if (fixed_split <= 0 && s > 1 && tiles * s > wave) continue;
            const double t = tile_cost(tiles, width, s, nkb, bytes, wave);
            if (best_t < 0.0 || t < best_t) {
                best_t = t;
                best = {cfg, width, s};
            }
        }
    };
    if (with_swap)
        for (int w : {16, 32, 64, 128, 256}) consider(HGEMM_SM100_CFG_SWAPAB, w, cdiv(n, 128) * cdiv(m, w), *swap_of_width(w).k);
    if (with_wide) consider(HGEMM_SM100_CFG_SPLITK_128x256, 256, cdiv(m, 128) * cdiv(n, 256), g_splitk_256);
    return best;
}

// plan_tiles_uncached, memoised per thread (it is evaluated on every call).
TilePlan plan_tiles(int64_t m, int64_t n, int64_t k, int sms, int max_split, bool with_swap, bool with_wide,
                    int32_t fixed_split) {
    struct Key {
        int64_t m, n, k;
        int32_t flags;
        bool operator==(const Key& o) const { return m == o.m && n == o.n && k == o.k && flags == o.flags; }
    };
    struct KeyHash {
        size_t operator()(const Key& x) const {
            size_t h = static_cast<size_t>(x.m) * 0x9E3779B97F4A7C15ull;
            h ^= static_cast<size_t>(x.n) * 0xC2B2AE3D27D4EB4Full + (h << 6) + (h >> 2);
            h ^= static_cast<size_t>(x.k) * 0x165667B19E3779F9ull + (h << 6) + (h >> 2);
            return h ^ static_cast<size_t>(x.flags);
        }
    };
    thread_local std::unordered_map<Key, TilePlan, KeyHash> cache;
    int dev = 0;
    (void)cudaGetDevice(&dev);
    const Key key{m, n, k,
                  (fixed_split << 16) | (dev << 4) | (with_swap ? 1 : 0) | (with_wide ? 2 : 0)};
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    const TilePlan tp = plan_tiles_uncached(m, n, k, sms, max_split, with_swap, with_wide, fixed_split);
    if (cache.size() >= 4096) cache.clear();
    cache.emplace(key, tp);
    return tp;
}

// Swapped-tile width for (m, n, k) at K split `split` (the cheapest).
SwapChoice swap_choice(int64_t m, int64_t n, int64_t k, int32_t split, int sms, int max_split) {
    return swap_of_width(plan_tiles(m, n, k, sms, max_split, true, false, split > 0 ? split : 1).width);
}

// Columns of C: n, or n / 2 with the SwiGLU epilogue.
int64_t out_cols(const HgemmSm100Args& a) { return (a.epilogue & HGEMM_SM100_EPI_SILU_MUL) ? a.n / 2 : a.n; }

int check_args(const HgemmSm100Args* a) {
    if (a == nullptr || a->a == nullptr || a->b == nullptr || a->c == nullptr)
        return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    if (a->m <= 0 || a->n <= 0 || a->k <= 0) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    const int64_t lim = (int64_t{1} << 31) - 1;
    if (a->m > lim || a->n > lim || a->k > lim) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    const int32_t epi = a->epilogue;
    const bool silu = (epi & HGEMM_SM100_EPI_SILU_MUL) != 0;
    if (a->lda < a->k || a->ldb < a->n || a->ldc < out_cols(*a)) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    if (epi & ~(HGEMM_SM100_EPI_BIAS | HGEMM_SM100_EPI_RESIDUAL | HGEMM_SM100_EPI_SILU_MUL))
        return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    if (epi != 0 && (a->flags & HGEMM_SM100_FLAG_OUT_F32)) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    if ((epi & HGEMM_SM100_EPI_BIAS) && a->bias == nullptr) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    if ((epi & HGEMM_SM100_EPI_RESIDUAL) && (a->residual == nullptr || a->ldr < a->n || silu))
        return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    if (silu && a->n % 2 != 0) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    if (a->config < 0 || a->config >= HGEMM_SM100_CFG_COUNT) return HGEMM_SM100_ERR_UNKNOWN_CONFIG;
    if (a->split_k < 0 || a->split_k > kMaxSplit) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    return HGEMM_SM100_OK;
}

// Raster group height (tile rows) of the CTA-pair kernels. A wave of P pair
// tiles spans about g rows and P / g columns of 256 x 256 tiles; the next
// wave of the same group re-reads those A rows, and every group re-reads all
// of B. Taller groups read B fewer times but push the previous wave's A rows
// further back in L2: the tallest of 8, 16, 32 whose one-wave footprint,
// (g + P / g) panels of 256 x K halves, stays within 48 MB (what kept the
// reuse in L2 when timed; 8 when none does, e.g. K = 8192).
int pair_group_m(int32_t cfg, int64_t m, int64_t k, int pairs) {
    int g = 8;
    if (cfg != HGEMM_SM100_CFG_PAIR_256x256 && cfg != HGEMM_SM100_CFG_STREAMK_PAIR_256x256) return g;
    const double panel = 512.0 * static_cast<double>(k);
    for (int h : {16, 32})
        if (h <= cdiv(m, 256) && (h + static_cast<double>(pairs) / h) * panel <= 48e6) g = h;
    return g;
}

// Stream-K configurations: tile geometry, grid and workspace of one launch.
struct StreamKPlan {
    KernelEntry* k = nullptr;
    int bnm = 0;
    bool swap = false;
    int64_t tiles = 0, kb = 0;
    int grid = 0;
    int streamk = 0;         // tiles split into K ranges (the last ones); 0 = none
    size_t slot_bytes = 0;   // one FP32 partial tile
    size_t bytes = 0;        // partial slots + flags
};

bool is_streamk(int32_t cfg) {
    return cfg == HGEMM_SM100_CFG_STREAMK_128x256 || cfg == HGEMM_SM100_CFG_STREAMK_SWAPAB ||
           cfg == HGEMM_SM100_CFG_STREAMK_PAIR_256x256;
}

StreamKPlan plan_streamk(int32_t cfg, int64_t m, int64_t n, int64_t k, int sms) {
    StreamKPlan sp;
    if (cfg == HGEMM_SM100_CFG_STREAMK_PAIR_256x256) {
        // Pairs of CTAs (grid = 2 x pairs), one 128-row half of a 256 x 256
        // partial tile per CTA slot, one flag per CTA.
        const int pairs = sms / 2;
        sp.k = &g_pair_sk_256;
        sp.bnm = 256;
        sp.tiles = cdiv(m, 256) * cdiv(n, 256);
        sp.kb = cdiv(k, kBlockK);
        const int64_t rem = sp.tiles % pairs;
        sp.streamk = (sp.tiles >= pairs && rem != 0) ? static_cast<int>(rem + pairs) : 0;
        sp.grid = 2 * static_cast<int>(sp.tiles < pairs ? sp.tiles : pairs);
        sp.slot_bytes = static_cast<size_t>(128) * 256 * 4;
        sp.bytes = sp.streamk ? static_cast<size_t>(sp.grid) * (sp.slot_bytes + 8) + 512 : 0;
        return sp;
    }
    if (cfg == HGEMM_SM100_CFG_STREAMK_SWAPAB) {
        sp.swap = true;
        if (m <= 16) { sp.bnm = 16; sp.k = &g_sk_swap_16; }
        else if (m <= 32) { sp.bnm = 32; sp.k = &g_sk_swap_32; }
        else if (m <= 64) { sp.bnm = 64; sp.k = &g_sk_swap_64; }
        else { sp.bnm = 128; sp.k = &g_sk_swap_128; }
        sp.tiles = cdiv(n, 128) * cdiv(m, sp.bnm);
    } else {
        sp.bnm = 256;
        sp.k = &g_sk_256;
        sp.tiles = cdiv(m, 128) * cdiv(n, 256);
    }
    sp.kb = cdiv(k, kBlockK);
    // Whole tiles in waves; when the last wave is partial, the last
    // (remainder + one full wave) tiles are split into equal K ranges, each
    // spanning at least one tile (so a split tile has exactly one producer).
    // With fewer tiles than SMs the ranges would be shorter than a tile:
    // whole tiles only (the split-K configurations cover that regime).
    const int64_t rem = sp.tiles % sms;
    sp.streamk = (sp.tiles >= sms && rem != 0) ? static_cast<int>(rem + sms) : 0;
    sp.grid = static_cast<int>(sp.tiles < sms ? sp.tiles : sms);
    sp.slot_bytes = static_cast<size_t>(128) * sp.bnm * 4;
    sp.bytes = sp.streamk ? static_cast<size_t>(sp.grid) * (sp.slot_bytes + 8) + 512 : 0;
    return sp;
}

// Split-K tile kernels: workspace for exchanging FP32 partial tiles, one slot
// per CTA (0 when there is no split). Without it the partials go through
// distributed shared memory, which is also the faster transport for tiles of
// at most 128 columns (partials up to 64 KB per CTA: remote stores plus one
// cluster barrier beat the two L2 round trips); the workspace serves the
// 256-column tiles (128 KB partials).
bool is_tile_cfg(int32_t cfg) {
    return cfg == HGEMM_SM100_CFG_SPLITK_128x128 || cfg == HGEMM_SM100_CFG_SPLITK_128x256 ||
           cfg == HGEMM_SM100_CFG_GENERIC_128x128 || cfg == HGEMM_SM100_CFG_SWAPAB;
}

size_t exchange_bytes(int32_t cfg, int64_t m, int64_t n, int64_t k, int32_t split, int sms, int max_split) {
    if (!is_tile_cfg(cfg) || split <= 1) return 0;
    int64_t ctas;
    size_t slot;
    if (cfg == HGEMM_SM100_CFG_SWAPAB) {
        const int bnm = swap_choice(m, n, k, split, sms, max_split).bnm;
        if (bnm <= 128) return 0;
        ctas = cdiv(n, 128) * cdiv(m, bnm);
        slot = static_cast<size_t>(128) * bnm * 4;
    } else {
        const int bn = cfg == HGEMM_SM100_CFG_SPLITK_128x256 ? 256 : 128;
        if (bn <= 128) return 0;
        ctas = cdiv(m, 128) * cdiv(n, bn);
        slot = static_cast<size_t>(128) * (bn + 4) * 4;
    }
    return static_cast<size_t>(ctas) * split * slot;
}

// Bytes of the kernel's own workspace region (after any staging buffers).
size_t region_need(int32_t cfg, int32_t split, int64_t m, int64_t n, int64_t k, int sms, int max_split) {
    if (is_streamk(cfg)) return plan_streamk(cfg, m, n, k, sms).bytes;
    return exchange_bytes(cfg, m, n, k, split, sms, max_split);
}

std::atomic<uint64_t> g_epoch_counter{0};

// A value no earlier launch of this process used (and, with the random base,
// none of another process): stale flags in a reused workspace never match.
uint64_t next_epoch() {
    static const uint64_t base = [] {
        std::random_device rd;
        return (static_cast<uint64_t>(rd()) << 32) ^ static_cast<uint64_t>(rd()) ^ 0x9E3779B97F4A7C15ull;
    }();
    uint64_t e = base + 0xD1B54A32D192ED03ull * (g_epoch_counter.fetch_add(1) + 1);
    return e == 0 ? 1 : e;
}

// Operand staging: TMA needs 16-byte-aligned bases and row pitches that are
// multiples of 8 halves (16 bytes). Operands breaking this are copied into
// padded, aligned buffers carved from the caller's workspace.
struct Staging {
    bool a = false, b = false, c = false;
    int64_t lda = 0, ldb = 0, ldc = 0;      // pitches of the staged copies
    size_t off_a = 0, off_b = 0, off_c = 0, total = 0;
};

constexpr size_t kStageAlign = 256;

size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

bool fp16_tma_ok(const void* ptr, int64_t ld) {
    return reinterpret_cast<uintptr_t>(ptr) % 16 == 0 && ld % 8 == 0;
}

Staging plan_staging(const HgemmSm100Args& a) {
    Staging st;
    if (a.config == HGEMM_SM100_CFG_GENERIC_128x128) return st;
    st.a = !fp16_tma_ok(a.a, a.lda);
    st.b = !fp16_tma_ok(a.b, a.ldb);
    const bool out_f32 = (a.flags & HGEMM_SM100_FLAG_OUT_F32) != 0;
    // A ragged FP16 C is computed into an aligned copy (16-byte epilogue
    // stores) and copied out; an FP32 C is never staged.
    st.c = !out_f32 && !fp16_tma_ok(a.c, a.ldc);
    size_t off = 0;
    if (st.a) {
        st.lda = static_cast<int64_t>(align_up(a.k, 8));
        st.off_a = off;
        off = align_up(off + static_cast<size_t>(a.m) * st.lda * 2, kStageAlign);
    }
    if (st.b) {
        st.ldb = static_cast<int64_t>(align_up(a.n, 8));
        st.off_b = off;
        off = align_up(off + static_cast<size_t>(a.k) * st.ldb * 2, kStageAlign);
    }
    if (st.c) {
        st.ldc = static_cast<int64_t>(align_up(out_cols(a), 8));
        st.off_c = off;
        off = align_up(off + static_cast<size_t>(a.m) * st.ldc * 2, kStageAlign);
    }
    st.total = off;
    return st;
}

bool staging_usable(const HgemmSm100Args& a, const Staging& st) {
    return st.total > 0 && a.workspace != nullptr && a.workspace_bytes >= st.total &&
           reinterpret_cast<uintptr_t>(a.workspace) % kStageAlign == 0;
}

// Configuration and K split for `a`. With assume_workspace the caller is
// taken to provide every workspace the result needs (used to size it);
// otherwise the workspace in `a` decides whether staging and stream-K apply.
int resolve_cfg(const HgemmSm100Args& a, const DeviceInfo& dev, bool assume_workspace, int32_t* cfg_out,
                int32_t* split_out) {
    int32_t cfg = a.config;
    const int64_t nkb = cdiv(a.k, kBlockK);
    const int sms = dev.sms > 0 ? dev.sms : 148;
    const Staging st = plan_staging(a);
    const bool ab_ready = !(st.a || st.b) || assume_workspace || staging_usable(a, st);
    if (!ab_ready) {
        cfg = HGEMM_SM100_CFG_GENERIC_128x128;
    } else if (cfg == HGEMM_SM100_CFG_AUTO) {
        // At least one tile per SM: persistent waves (+ a stream-K split tail).
        // Fewer tiles than SMs: one tile per CTA, K split across a cluster.
        const int64_t wide_tiles = cdiv(a.m, 128) * cdiv(a.n, 256);
        if (a.m <= 128 && cdiv(a.n, 128) >= sms) {
            cfg = HGEMM_SM100_CFG_STREAMK_SWAPAB;
        } else if (a.m <= 2048 && wide_tiles < sms) {
            // Few tiles: the cost model picks the tile width and K split.
            const TilePlan tp = plan_tiles(a.m, a.n, a.k, sms, dev.max_cluster, true, a.m > 128, a.split_k);
            *cfg_out = tp.cfg;
            *split_out = tp.split;
            return HGEMM_SM100_OK;
        } else {
            // At least one wave: the persistent kernel runs whole tiles; its
            // partial last wave leaves SMs idle for (1 - fill) of a wave.
            // Stream-K spreads that tail but pays its partial-tile fixup
            // (about 6 us). It is used below 8 waves when the idle time it
            // removes (a 128 x 256 tile's K block takes about 0.30 us) is
            // larger than that.
            const int64_t tiles = cdiv(a.m, 128) * cdiv(a.n, 256);
            const int64_t waves = tiles / sms, rem = tiles % sms;
            const double idle_us = rem == 0 ? 0.0
                                            : (1.0 - static_cast<double>(rem) / sms) * 0.30 * static_cast<double>(nkb);
            const bool spread_tail = waves < 8 && idle_us > 6.0;
            cfg = tiles < sms      ? HGEMM_SM100_CFG_SPLITK_128x256
                  : spread_tail    ? HGEMM_SM100_CFG_STREAMK_128x256
                                   : HGEMM_SM100_CFG_PERSISTENT_128x256;
            // CTA pairs on 256 x 256 tiles: each SM streams 32 instead of
            // 48 KB per K block for the same MMA work, which ran 5-7 % faster
            // per tile than the 1-CTA kernel on every large FP16-output shape
            // measured and 7-20 % faster with FP32 output (the tensor-parallel
            // down-projection partials, 8192 x 2560 x 2432 .. 9728); they win
            // unless their coarser tiles leave a worse last wave. Times below in 128 x 256 K blocks of one SM;
            // the stream-K split tail is charged what it cost when timed
            // against whole-tile waves (25 K blocks + 0.4 per K block of a
            // tile), and the pairs replace it only when 3 % ahead.
            if (tiles >= sms) {
                const int64_t pairs = sms / 2;
                const int64_t tiles2 = cdiv(a.m, 256) * cdiv(a.n, 256);
                const double kb = static_cast<double>(nkb);
                const double t_pair = static_cast<double>(cdiv(tiles2, pairs)) * kb * 0.93;
                double t_best = spread_tail ? static_cast<double>(tiles) / sms * kb + 25.0 + 0.4 * kb
                                            : static_cast<double>(cdiv(tiles, sms)) * kb;
                if (spread_tail ? t_pair < 0.97 * t_best : t_pair <= t_best) {
                    cfg = HGEMM_SM100_CFG_PAIR_256x256;
                    t_best = t_pair;
                }
                // Stream-K over pairs: whole pair-tile waves, then the partial
                // last wave's K blocks spread over every pair; its fixup cost
                // measured 10 + 0.47 K blocks. It pays off when the last wave
                // of 256 x 256 tiles is nearly empty.
                if (tiles2 >= pairs && tiles2 % pairs != 0) {
                    const double t_psk = static_cast<double>(tiles2) / pairs * kb * 0.93 + 10.0 + 0.47 * kb;
                    if (t_psk < 0.97 * t_best) cfg = HGEMM_SM100_CFG_STREAMK_PAIR_256x256;
                }
            }
            // Narrow tiles when they (with their K split) fill the SMs in one
            // wave: the same MMA time per K block, half the partial tile to
            // exchange, or no split at all.
            if (cfg == HGEMM_SM100_CFG_SPLITK_128x256) {
                const int64_t narrow = cdiv(a.m, 128) * cdiv(a.n, 128);
                const int64_t ctas = narrow * choose_split(narrow, nkb, sms, dev.max_cluster);
                if (narrow <= sms && 5 * ctas >= 4 * static_cast<int64_t>(sms)) cfg = HGEMM_SM100_CFG_SPLITK_128x128;
            }
        }
    }
    if (cfg == HGEMM_SM100_CFG_STREAMK_SWAPAB && a.m > 128) cfg = HGEMM_SM100_CFG_STREAMK_128x256;
    if (is_streamk(cfg) && !assume_workspace) {
        const StreamKPlan sp = plan_streamk(cfg, a.m, a.n, a.k, sms);
        const size_t need = align_up(st.total, kStageAlign) + sp.bytes;
        const size_t have = a.workspace != nullptr ? a.workspace_bytes : 0;
        if (sp.bytes > 0 && have < need)
            cfg = cfg == HGEMM_SM100_CFG_STREAMK_SWAPAB        ? HGEMM_SM100_CFG_SWAPAB
                  : cfg == HGEMM_SM100_CFG_STREAMK_PAIR_256x256 ? HGEMM_SM100_CFG_PAIR_256x256
                                                                : HGEMM_SM100_CFG_PERSISTENT_128x256;
    }

    int32_t split = 1;
    if (cfg == HGEMM_SM100_CFG_SPLITK_128x128 || cfg == HGEMM_SM100_CFG_SPLITK_128x256 ||
        cfg == HGEMM_SM100_CFG_GENERIC_128x128 || cfg == HGEMM_SM100_CFG_SWAPAB) {
        int64_t base;
        int per_sm = 1;
        if (cfg == HGEMM_SM100_CFG_SWAPAB && a.split_k <= 0) {
            // Width and split from the cost model (the split already fits
            // the clusters that can be resident).
            *cfg_out = cfg;
            *split_out = plan_tiles(a.m, a.n, a.k, sms, dev.max_cluster, true, false, 0).split;
            return HGEMM_SM100_OK;
        }
        if (cfg == HGEMM_SM100_CFG_SWAPAB) {
            const SwapChoice sc = swap_choice(a.m, a.n, a.k, a.split_k, sms, dev.max_cluster);
            base = cdiv(a.n, 128) * cdiv(a.m, sc.bnm);
            per_sm = sc.per_sm;
        } else if (cfg == HGEMM_SM100_CFG_SPLITK_128x256) {
            base = cdiv(a.m, 128) * cdiv(a.n, 256);
        } else {
            base = cdiv(a.m, 128) * cdiv(a.n, 128);
        }
        split = a.split_k > 0 ? a.split_k : choose_split(base, nkb, sms * per_sm, dev.max_cluster);
        if (split > nkb) split = static_cast<int32_t>(nkb);
        if (split < 1) split = 1;
        if (a.split_k <= 0 && split > 1) {
            KernelEntry* k = cfg == HGEMM_SM100_CFG_SWAPAB ? swap_choice(a.m, a.n, a.k, split, sms, dev.max_cluster).k
                             : cfg == HGEMM_SM100_CFG_SPLITK_128x256 ? &g_splitk_256
                             : cfg == HGEMM_SM100_CFG_SPLITK_128x128 ? &g_splitk_128
                                                                     : &g_generic_128;
            int devid = 0;
            if (cudaGetDevice(&devid) == cudaSuccess) split = fit_split(*k, devid, base, split);
        }
    }
    *cfg_out = cfg;
    *split_out = split;
    return HGEMM_SM100_OK;
}

int resolve(const HgemmSm100Args& a, const DeviceInfo& dev, int32_t* cfg_out, int32_t* split_out) {
    return resolve_cfg(a, dev, false, cfg_out, split_out);
}

int launch(const KernelEntry& k, dim3 grid, int cluster_z, const CUtensorMap& m0, const CUtensorMap& m1,
           const CUtensorMap& m2, const GemmParams& p, cudaStream_t stream, int cluster_x = 1,
           bool cooperative = false) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = k.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[3];
    unsigned n = 0;
    if (cluster_z > 1 || cluster_x > 1) {
        attr[n].id = cudaLaunchAttributeClusterDimension;
        attr[n].val.clusterDim.x = static_cast<unsigned>(cluster_x);
        attr[n].val.clusterDim.y = 1;
        attr[n].val.clusterDim.z = static_cast<unsigned>(cluster_z);
        ++n;
    }
    if (cooperative) {
        // Stream-K finishers wait for other CTAs: all must be resident.
        attr[n].id = cudaLaunchAttributeCooperative;
        attr[n].val.cooperative = 1;
        ++n;
    } else {
        // Programmatic dependent launch: the kernel's set-up overlaps the
        // previous kernel of the stream (the kernels wait for it before
        // touching global memory).
        attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n].val.programmaticStreamSerializationAllowed = 1;
        ++n;
    }
    if (n > 0) {
        cfg.attrs = attr;
        cfg.numAttrs = n;
    }
    const KernelFn fn = reinterpret_cast<KernelFn>(const_cast<void*>(k.fn));
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, m0, m1, m2, p);
    return e == cudaSuccess ? HGEMM_SM100_OK : HGEMM_SM100_ERR_LAUNCH;
}

int launch_copy(const __half* src, int64_t ld_src, __half* dst, int64_t ld_dst, int64_t rows,
                int64_t cols, bool dst_aligned, int sms, cudaStream_t stream) {
    // ~8 blocks of 256 threads per SM in flight; x covers a row's chunks.
    int64_t bx = cdiv(cdiv(cols, 8), 256);
    if (bx > 64) bx = 64;
    int64_t by = cdiv(static_cast<int64_t>(sms) * 8, bx);
    if (by > rows) by = rows;
    if (by > 65535) by = 65535;
    const dim3 grid(static_cast<unsigned>(bx), static_cast<unsigned>(by), 1);
    if (dst_aligned)
        copy_rows_kernel<true><<<grid, 256, 0, stream>>>(src, ld_src, dst, ld_dst, rows, cols);
    else
        copy_rows_kernel<false><<<grid, 256, 0, stream>>>(src, ld_src, dst, ld_dst, rows, cols);
    return cudaGetLastError() == cudaSuccess ? HGEMM_SM100_OK : HGEMM_SM100_ERR_LAUNCH;
}

// Launches the resolved configuration on operands that TMA can describe
// (or, for the generic configuration, on any operands).
int run_core(const HgemmSm100Args& a, int32_t cfg, int32_t split, const DeviceInfo& dev, int devid,
             cudaStream_t stream, uint8_t* region, size_t region_bytes,
             const HgemmSm100Scatter* sc = nullptr) {
    int rc = HGEMM_SM100_OK;
    GemmParams p{};
    p.a = static_cast<const __half*>(a.a);
    p.b = static_cast<const __half*>(a.b);
    p.c = a.c;
    p.m = static_cast<int>(a.m);
    p.n = static_cast<int>(a.n);
    p.k = static_cast<int>(a.k);
    p.lda = a.lda;
    p.ldb = a.ldb;
    p.ldc = a.ldc;
    p.out_f32 = (a.flags & HGEMM_SM100_FLAG_OUT_F32) ? 1 : 0;
    p.vec_ok = (reinterpret_cast<uintptr_t>(a.c) % 16 == 0) && (a.ldc % 8 == 0);
    p.group_m = 16;
    p.inject = (a.flags & HGEMM_SM100_FLAG_TEST_INJECT_TX) ? 1 : 0;
    p.status = a.status != nullptr ? a.status : dev.status_word;
    p.timeout_ns = a.timeout_ns != 0 ? a.timeout_ns : kDefaultTimeoutNs;
    p.epi = a.epilogue;
    p.bias = static_cast<const __half*>(a.bias);
    p.residual = static_cast<const __half*>(a.residual);
    p.ldr = a.ldr;
    if (sc != nullptr) {
        p.sc_ranks = sc->ranks;
        p.sc_rank = sc->rank;
        p.sc_rows = static_cast<int>(sc->rows_per_rank);
        p.sc_ld = sc->ld_dest;
        bool aligned = sc->ld_dest % 8 == 0;
        for (int q = 0; q < sc->ranks; ++q) {
            p.sc_dest[q] = static_cast<float*>(sc->dest[q]);
            aligned = aligned && reinterpret_cast<uintptr_t>(sc->dest[q]) % 16 == 0;
        }
        p.vec_ok = aligned;
        // Bulk row copies: 16-byte-aligned rows (aligned above) of whole 16-byte
        // pieces; the persistent and CTA-pair kernels use them.
        p.sc_bulk = aligned && a.n % 4 == 0 &&
                    (cfg == HGEMM_SM100_CFG_PERSISTENT_128x256 || cfg == HGEMM_SM100_CFG_PERSISTENT_128x128 ||
                     cfg == HGEMM_SM100_CFG_PAIR_256x256 || cfg == HGEMM_SM100_CFG_PAIR_256x128 ||
                     cfg == HGEMM_SM100_CFG_PAIR_128x256 || cfg == HGEMM_SM100_CFG_PAIR_128x128);
    }
    p.epi_vec = (p.epi & HGEMM_SM100_EPI_BIAS ? reinterpret_cast<uintptr_t>(a.bias) % 16 == 0 : true) &&
                (p.epi & HGEMM_SM100_EPI_RESIDUAL
                     ? reinterpret_cast<uintptr_t>(a.residual) % 16 == 0 && a.ldr % 8 == 0
                     : true);

    CUtensorMap map_k, map_mn, map_c;
    std::memset(&map_k, 0, sizeof(map_k));
    std::memset(&map_mn, 0, sizeof(map_mn));
    std::memset(&map_c, 0, sizeof(map_c));
    // TMA-store epilogue (persistent and pair kernels): FP16 C whose base and
    // pitch TMA can describe; boxes of 32 rows x 64 columns.
    // Swapped tile kernels store [kChunk rows x 32 columns] boxes, unswizzled.
    // With the SwiGLU epilogue (half-width C) only the swapped tiles (box_cols
    // 32 -> 16 output columns) use TMA stores; the others store from registers.
    auto prepare_store = [&](uint32_t box_cols = 64, uint32_t box_rows = 32, bool swizzle = true) -> int {
        const bool silu = (p.epi & HGEMM_SM100_EPI_SILU_MUL) != 0;
        if (!p.vec_ok || p.out_f32 || (silu && box_cols != 32)) return HGEMM_SM100_OK;
        const int r = tensor_map(&map_c, a.c, static_cast<uint64_t>(out_cols(a)), static_cast<uint64_t>(a.m),
                                 static_cast<uint64_t>(a.ldc), silu ? box_cols / 2 : box_cols, box_rows, swizzle);
        if (r == HGEMM_SM100_OK) p.tma_store = 1;
        return r;
    };
    // Split-K partial exchange through the workspace when the caller gave one.
    if (split > 1 && region != nullptr &&
        region_bytes >= exchange_bytes(cfg, a.m, a.n, a.k, split, dev.sms, dev.max_cluster))
        p.partials = reinterpret_cast<float*>(region);
    const uint64_t M = a.m, N = a.n, K = a.k;

    switch (cfg) {
        case HGEMM_SM100_CFG_PERSISTENT_128x256:
        case HGEMM_SM100_CFG_PERSISTENT_128x128: {
            const bool wide = cfg == HGEMM_SM100_CFG_PERSISTENT_128x256;
            KernelEntry& k = wide ? g_persist_256 : g_persist_128;
            const int bn = wide ? 256 : 128;
            if ((rc = tensor_map(&map_k, a.a, K, M, a.lda, 64, 128)) != HGEMM_SM100_OK) return rc;
            if ((rc = tensor_map(&map_mn, a.b, N, K, a.ldb, 64, 64)) != HGEMM_SM100_OK) return rc;
            if ((rc = prepare_store()) != HGEMM_SM100_OK) return rc;
            if ((rc = prepare_kernel(k, devid)) != HGEMM_SM100_OK) return rc;
            const int64_t tiles = cdiv(a.m, 128) * cdiv(a.n, bn);
            const int64_t grid = tiles < dev.sms ? tiles : dev.sms;
            return launch(k, dim3(static_cast<unsigned>(grid), 1, 1), 1, map_k, map_mn, map_c, p, stream);
        }
        case HGEMM_SM100_CFG_PAIR_256x256:
        case HGEMM_SM100_CFG_PAIR_256x128:
        case HGEMM_SM100_CFG_PAIR_128x256:
        case HGEMM_SM100_CFG_PAIR_128x128: {
            const int tm = (cfg == HGEMM_SM100_CFG_PAIR_256x256 || cfg == HGEMM_SM100_CFG_PAIR_256x128) ? 256 : 128;
            const int tn = (cfg == HGEMM_SM100_CFG_PAIR_256x256 || cfg == HGEMM_SM100_CFG_PAIR_128x256) ? 256 : 128;
            KernelEntry& k = cfg == HGEMM_SM100_CFG_PAIR_256x256   ? g_pair_256
                             : cfg == HGEMM_SM100_CFG_PAIR_256x128 ? g_pair_128
                             : cfg == HGEMM_SM100_CFG_PAIR_128x256 ? g_pair_m128_256
                                                                   : g_pair_m128_128;
            if ((rc = tensor_map(&map_k, a.a, K, M, a.lda, 64, static_cast<uint32_t>(tm / 2))) != HGEMM_SM100_OK)
                return rc;
            if ((rc = tensor_map(&map_mn, a.b, N, K, a.ldb, 64, 64)) != HGEMM_SM100_OK) return rc;
            if ((rc = prepare_store()) != HGEMM_SM100_OK) return rc;
            if ((rc = prepare_kernel(k, devid)) != HGEMM_SM100_OK) return rc;
            const int64_t tiles = cdiv(a.m, tm) * cdiv(a.n, tn);
            const int64_t pairs_max = dev.sms / 2;
            const int64_t pairs = tiles < pairs_max ? tiles : pairs_max;
            p.group_m = pair_group_m(cfg, a.m, a.k, static_cast<int>(pairs_max));
            return launch(k, dim3(static_cast<unsigned>(2 * pairs), 1, 1), 1, map_k, map_mn, map_c, p, stream, 2);
        }
        case HGEMM_SM100_CFG_SPLITK_128x128:
        case HGEMM_SM100_CFG_SPLITK_128x256: {
            const bool wide = cfg == HGEMM_SM100_CFG_SPLITK_128x256;
            KernelEntry& k = wide ? g_splitk_256 : g_splitk_128;
            const int bn = wide ? 256 : 128;
            if ((rc = tensor_map(&map_k, a.a, K, M, a.lda, 64, 128)) != HGEMM_SM100_OK) return rc;
            if ((rc = tensor_map(&map_mn, a.b, N, K, a.ldb, 64, 64)) != HGEMM_SM100_OK) return rc;
            if (split == 1 && (rc = prepare_store()) != HGEMM_SM100_OK) return rc;
            if ((rc = prepare_kernel(k, devid)) != HGEMM_SM100_OK) return rc;
            const dim3 grid(static_cast<unsigned>(cdiv(a.m, 128)), static_cast<unsigned>(cdiv(a.n, bn)),
                            static_cast<unsigned>(split));
            return launch(k, grid, split, map_k, map_mn, map_c, p, stream);
        }
        case HGEMM_SM100_CFG_SWAPAB: {
            const SwapChoice sc = swap_choice(a.m, a.n, a.k, split, dev.sms, dev.max_cluster);
            if ((rc = tensor_map(&map_k, a.a, K, M, a.lda, 64, static_cast<uint32_t>(sc.bnm))) !=
                HGEMM_SM100_OK)
                return rc;
            if ((rc = tensor_map(&map_mn, a.b, N, K, a.ldb, 64, 64)) != HGEMM_SM100_OK) return rc;
            if (split == 1 && (rc = prepare_store(32, sc.bnm >= 32 ? 32 : 16, false)) != HGEMM_SM100_OK) return rc;
            if ((rc = prepare_kernel(*sc.k, devid)) != HGEMM_SM100_OK) return rc;
            const dim3 grid(static_cast<unsigned>(cdiv(a.n, 128)),
                            static_cast<unsigned>(cdiv(a.m, sc.bnm)), static_cast<unsigned>(split));
            return launch(*sc.k, grid, split, map_k, map_mn, map_c, p, stream);
        }
        case HGEMM_SM100_CFG_STREAMK_PAIR_256x256: {
            const StreamKPlan sp = plan_streamk(cfg, a.m, a.n, a.k, dev.sms);
            if ((rc = tensor_map(&map_k, a.a, K, M, a.lda, 64, 128)) != HGEMM_SM100_OK) return rc;
            if ((rc = tensor_map(&map_mn, a.b, N, K, a.ldb, 64, 64)) != HGEMM_SM100_OK) return rc;
            if ((rc = prepare_store()) != HGEMM_SM100_OK) return rc;
            if ((rc = prepare_kernel(*sp.k, devid)) != HGEMM_SM100_OK) return rc;
            p.streamk = sp.streamk;
            p.group_m = pair_group_m(cfg, a.m, a.k, dev.sms / 2);
            if (sp.streamk) {
                if (region == nullptr || region_bytes < sp.bytes) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
                p.partials = reinterpret_cast<float*>(region);
                p.flags = reinterpret_cast<unsigned long long*>(region +
                                                                static_cast<size_t>(sp.grid) * sp.slot_bytes);
                p.epoch = next_epoch();
            }
            return launch(*sp.k, dim3(static_cast<unsigned>(sp.grid), 1, 1), 1, map_k, map_mn, map_c, p, stream, 2);
        }
        case HGEMM_SM100_CFG_STREAMK_128x256:
        case HGEMM_SM100_CFG_STREAMK_SWAPAB: {
            const StreamKPlan sp = plan_streamk(cfg, a.m, a.n, a.k, dev.sms);
            if (sp.swap) {
                if ((rc = tensor_map(&map_k, a.a, K, M, a.lda, 64, static_cast<uint32_t>(sp.bnm))) !=
                    HGEMM_SM100_OK)
                    return rc;
            } else if ((rc = tensor_map(&map_k, a.a, K, M, a.lda, 64, 128)) != HGEMM_SM100_OK) {
                return rc;
            }
            if ((rc = tensor_map(&map_mn, a.b, N, K, a.ldb, 64, 64)) != HGEMM_SM100_OK) return rc;
            if ((rc = sp.swap ? prepare_store(32, sp.bnm >= 32 ? 32 : 16, false) : prepare_store()) != HGEMM_SM100_OK)
                return rc;
            if ((rc = prepare_kernel(*sp.k, devid)) != HGEMM_SM100_OK) return rc;
            p.streamk = sp.streamk;
            p.group_m = sp.swap ? 1 : 16;
            if (sp.streamk) {
                if (region == nullptr || region_bytes < sp.bytes) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
                p.partials = reinterpret_cast<float*>(region);
                p.flags = reinterpret_cast<unsigned long long*>(region +
                                                                static_cast<size_t>(sp.grid) * sp.slot_bytes);
                p.epoch = next_epoch();
            }
            return launch(*sp.k, dim3(static_cast<unsigned>(sp.grid), 1, 1), 1, map_k, map_mn, map_c, p, stream, 1,
                          sp.streamk != 0);
        }
        case HGEMM_SM100_CFG_GENERIC_128x128: {
            if (split == 1 && (rc = prepare_store()) != HGEMM_SM100_OK) return rc;
            if ((rc = prepare_kernel(g_generic_128, devid)) != HGEMM_SM100_OK) return rc;
            const dim3 grid(static_cast<unsigned>(cdiv(a.m, 128)), static_cast<unsigned>(cdiv(a.n, 128)),
                            static_cast<unsigned>(split));
            return launch(g_generic_128, grid, split, map_k, map_mn, map_c, p, stream);
        }
        default:
            return HGEMM_SM100_ERR_UNKNOWN_CONFIG;
    }
}

}  // namespace

// ================================================================== C ABI ==

extern "C" int hgemm_sm100_resolve(const HgemmSm100Args* args, int32_t* config_out, int32_t* split_out) {
    int rc = check_args(args);
    if (rc != HGEMM_SM100_OK) return rc;
    if (config_out == nullptr || split_out == nullptr) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    const DeviceInfo* dev = nullptr;
    rc = device_info(&dev);
    if (rc != HGEMM_SM100_OK) return rc;
    return resolve(*args, *dev, config_out, split_out);
}

namespace {

int run_impl(const HgemmSm100Args* args, const HgemmSm100Scatter* sc, void* stream_ptr) {
    int rc = check_args(args);
    if (rc != HGEMM_SM100_OK) return rc;
    const DeviceInfo* dev = nullptr;
    rc = device_info(&dev);
    if (rc != HGEMM_SM100_OK) return rc;
    int devid = 0;
    cudaGetDevice(&devid);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);

    int32_t cfg = 0, split = 1;
    rc = resolve(*args, *dev, &cfg, &split);
    if (rc != HGEMM_SM100_OK) return rc;
    // A row scatter's FP32 rows leave through bulk copies in the epilogue; with
    // short K that epilogue weighs more in the CTA-pair kernel than in the
    // 1-CTA persistent one (8192 x 2560 partials, K = 1216 / 2432: pairs 10 % /
    // 3 % slower; K = 4864 and 8192 x 8192 partials, K = 3584 .. 14336: 3-6 %
    // faster), so `auto` keeps the 1-CTA kernel below K = 3072.
    if (sc != nullptr && args->config == HGEMM_SM100_CFG_AUTO && args->k < 3072 &&
        (cfg == HGEMM_SM100_CFG_PAIR_256x256 || cfg == HGEMM_SM100_CFG_STREAMK_PAIR_256x256))
        cfg = HGEMM_SM100_CFG_PERSISTENT_128x256;

    // Workspace layout: [staging buffers][kernel region: stream-K partial
    // slots + flags, or split-K exchange slots].
    const Staging st = plan_staging(*args);
    const bool staged = cfg != HGEMM_SM100_CFG_GENERIC_128x128 && staging_usable(*args, st);
    uint8_t* ws = static_cast<uint8_t*>(args->workspace);
    uint8_t* region = nullptr;
    size_t region_bytes = 0;
    const size_t region_off = align_up(staged ? st.total : 0, kStageAlign);
    if (ws != nullptr && reinterpret_cast<uintptr_t>(ws) % kStageAlign == 0 && args->workspace_bytes > region_off &&
        region_need(cfg, split, args->m, args->n, args->k, dev->sms, dev->max_cluster) > 0) {
        region = ws + region_off;
        region_bytes = static_cast<size_t>(args->workspace_bytes) - region_off;
    }

    if (!staged) return run_core(*args, cfg, split, *dev, devid, stream, region, region_bytes, sc);

    // Stage, run on the staged operands, copy a staged C back.
    HgemmSm100Args s = *args;
    if (st.a) {
        __half* dst = reinterpret_cast<__half*>(ws + st.off_a);
        if ((rc = launch_copy(static_cast<const __half*>(args->a), args->lda, dst, st.lda, args->m, args->k,
                              true, dev->sms, stream)) != HGEMM_SM100_OK)
            return rc;
        s.a = dst;
        s.lda = st.lda;
    }
    if (st.b) {
        __half* dst = reinterpret_cast<__half*>(ws + st.off_b);
        if ((rc = launch_copy(static_cast<const __half*>(args->b), args->ldb, dst, st.ldb, args->k, args->n,
                              true, dev->sms, stream)) != HGEMM_SM100_OK)
            return rc;
        s.b = dst;
        s.ldb = st.ldb;
    }
    if (st.c) {
        s.c = ws + st.off_c;
        s.ldc = st.ldc;
    }
    s.config = cfg;
    s.split_k = split;
    if ((rc = run_core(s, cfg, split, *dev, devid, stream, region, region_bytes, sc)) != HGEMM_SM100_OK) return rc;
    if (st.c)
        return launch_copy(static_cast<const __half*>(s.c), st.ldc, static_cast<__half*>(args->c), args->ldc,
                           args->m, out_cols(*args), false, dev->sms, stream);
    return HGEMM_SM100_OK;
}

}  // namespace

extern "C" int hgemm_sm100_run(const HgemmSm100Args* args, void* stream_ptr) {
    return run_impl(args, nullptr, stream_ptr);
}

// ============================================== tensor-parallel row scatter ==

extern "C" int hgemm_sm100_run_scatter(const HgemmSm100Args* args, const HgemmSm100Scatter* sc,
                                       void* stream_ptr) {
    if (args == nullptr || sc == nullptr) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    if (!(args->flags & HGEMM_SM100_FLAG_OUT_F32) || args->epilogue != 0) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    if (sc->ranks < 1 || sc->ranks > HGEMM_SM100_MAX_RANKS || sc->rank < 0 || sc->rank >= sc->ranks)
        return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    if (sc->rows_per_rank <= 0 || sc->rows_per_rank * sc->ranks != args->m || sc->ld_dest < args->n)
        return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    for (int q = 0; q < sc->ranks; ++q)
        if (sc->dest[q] == nullptr) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    return run_impl(args, sc, stream_ptr);
}

extern "C" int hgemm_sm100_reduce_slots(const void* slots, int32_t ranks, int64_t rows, int64_t cols,
                                        int64_t ld_slots, void* out, int64_t ld_out, void* stream_ptr) {
    return hgemm_sm100_reduce_slots_gather(slots, ranks, rows, cols, ld_slots, &out, 1, ld_out, stream_ptr);
}

extern "C" int hgemm_sm100_reduce_slots_gather(const void* slots, int32_t ranks, int64_t rows, int64_t cols,
                                               int64_t ld_slots, void* const* outs, int32_t n_outs, int64_t ld_out,
                                               void* stream_ptr) {
    if (slots == nullptr || outs == nullptr || n_outs < 1 || n_outs > HGEMM_SM100_MAX_RANKS || ranks < 1 ||
        ranks > HGEMM_SM100_MAX_RANKS || rows <= 0 || cols <= 0 || ld_slots < cols || ld_out < cols)
        return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    SlotOutputs o{};
    o.count = n_outs;
    bool out_aligned = true;
    for (int i = 0; i < n_outs; ++i) {
        if (outs[i] == nullptr) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
        o.ptr[i] = static_cast<__half*>(outs[i]);
        out_aligned = out_aligned && reinterpret_cast<uintptr_t>(outs[i]) % 8 == 0;
    }
    const DeviceInfo* dev = nullptr;
    const int rc = device_info(&dev);
    if (rc != HGEMM_SM100_OK) return rc;
    const bool vec = cols % 4 == 0 && ld_slots % 4 == 0 && ld_out % 4 == 0 &&
                     reinterpret_cast<uintptr_t>(slots) % 16 == 0 && out_aligned;
    const int64_t items = rows * (vec ? cols / 4 : cols);
    // HBM-bound: 8 blocks of 256 threads per SM, grid-stride.
    int64_t blocks = cdiv(items, 256);
    if (blocks > static_cast<int64_t>(dev->sms) * 8) blocks = static_cast<int64_t>(dev->sms) * 8;
    cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
    const float* src = static_cast<const float*>(slots);
    if (vec)
        reduce_slots_kernel<true><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, ranks, rows, cols,
                                                                                    ld_slots, o, ld_out);
    else
        reduce_slots_kernel<false><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(src, ranks, rows, cols,
                                                                                     ld_slots, o, ld_out);
    return cudaGetLastError() == cudaSuccess ? HGEMM_SM100_OK : HGEMM_SM100_ERR_LAUNCH;
}

extern "C" int hgemm_sm100_alloc_shared(uint64_t bytes, void** ptr_out) {
    if (ptr_out == nullptr || bytes == 0) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    *ptr_out = nullptr;
    return cudaMalloc(ptr_out, bytes) == cudaSuccess ? HGEMM_SM100_OK : HGEMM_SM100_ERR_CUDA;
}

extern "C" int hgemm_sm100_free_shared(void* ptr) {
    return cudaFree(ptr) == cudaSuccess ? HGEMM_SM100_OK : HGEMM_SM100_ERR_CUDA;
}

extern "C" int hgemm_sm100_ipc_handle(const void* ptr, void* handle_out) {
    if (ptr == nullptr || handle_out == nullptr) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "64-byte IPC handle");
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)) != cudaSuccess) return HGEMM_SM100_ERR_CUDA;
    std::memcpy(handle_out, &h, sizeof(h));
    return HGEMM_SM100_OK;
}

extern "C" int hgemm_sm100_ipc_open(const void* handle, void** ptr_out) {
    if (handle == nullptr || ptr_out == nullptr) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    *ptr_out = nullptr;
    return cudaIpcOpenMemHandle(ptr_out, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? HGEMM_SM100_OK
                                                                                          : HGEMM_SM100_ERR_CUDA;
}

extern "C" int hgemm_sm100_ipc_close(void* ptr) {
    return cudaIpcCloseMemHandle(ptr) == cudaSuccess ? HGEMM_SM100_OK : HGEMM_SM100_ERR_CUDA;
}

extern "C" size_t hgemm_sm100_workspace_size(const HgemmSm100Args* args) {
    if (check_args(args) != HGEMM_SM100_OK) return 0;
    const Staging st = plan_staging(*args);
    size_t total = st.total;
    const DeviceInfo* dev = nullptr;
    if (device_info(&dev) != HGEMM_SM100_OK) return total;
    int32_t cfg = 0, split = 0;
    resolve_cfg(*args, *dev, true, &cfg, &split);
    if (cfg == HGEMM_SM100_CFG_GENERIC_128x128) return 0;
    const size_t region = region_need(cfg, split, args->m, args->n, args->k, dev->sms, dev->max_cluster);
    if (region > 0) total = align_up(total, kStageAlign) + region;
    return total;
}

extern "C" int32_t hgemm_sm100_config_from_name(const char* name) {
    if (name == nullptr) return -1;
    for (int32_t i = 0; i < HGEMM_SM100_CFG_COUNT; ++i)
        if (std::strcmp(name, kConfigNames[i]) == 0) return i;
    return -1;
}

extern "C" const char* hgemm_sm100_config_name(int32_t config) {
    if (config < 0 || config >= HGEMM_SM100_CFG_COUNT) return nullptr;
    return kConfigNames[config];
}

extern "C" int32_t hgemm_sm100_num_configs(void) { return HGEMM_SM100_CFG_COUNT; }

extern "C" size_t hgemm_sm100_workspace_bytes(int32_t config, int64_t m, int64_t n, int64_t k) {
    if (m <= 0 || n <= 0 || k <= 0 || config < 0 || config >= HGEMM_SM100_CFG_COUNT) return 0;
    const DeviceInfo* dev = nullptr;
    if (device_info(&dev) != HGEMM_SM100_OK) return 0;
    // The configuration (auto resolved) and split chosen for aligned operands
    // when the caller gives every workspace asked for.
    HgemmSm100Args a{};
    static const uint8_t dummy[16] = {};
    a.a = a.b = dummy;
    a.c = const_cast<uint8_t*>(dummy);
    a.m = m;
    a.n = n;
    a.k = k;
    a.lda = align_up(static_cast<size_t>(k), 8);
    a.ldb = a.ldc = align_up(static_cast<size_t>(n), 8);
    a.config = config;
    int32_t cfg = 0, split = 0;
    if (resolve_cfg(a, *dev, true, &cfg, &split) != HGEMM_SM100_OK) return 0;
    return region_need(cfg, split, m, n, k, dev->sms, dev->max_cluster);
}

extern "C" const char* hgemm_sm100_status_string(int status) {
    switch (status) {
        case HGEMM_SM100_OK: return "ok";
        case HGEMM_SM100_ERR_INVALID_ARGUMENT: return "invalid argument";
        case HGEMM_SM100_ERR_UNKNOWN_CONFIG: return "unknown implementation";
        case HGEMM_SM100_ERR_UNSUPPORTED_DEVICE: return "device is not an sm_100 (B200) GPU";
        case HGEMM_SM100_ERR_LAUNCH: return "kernel launch failed";
        case HGEMM_SM100_ERR_PIPELINE_TIMEOUT: return "hgemm: pipeline timeout";
        case HGEMM_SM100_ERR_TENSOR_MAP: return "TMA descriptor encoding failed";
        case HGEMM_SM100_ERR_CUDA: return "CUDA runtime error";
        case HGEMM_SM100_ERR_SCRATCH_LIMIT:
            return "problem needs more scratch than the static buffer (HGEMM_SM100_STATIC_SCRATCH_BYTES)";
        case HGEMM_SM100_ERR_DEBUG_BOUNDS: return "hgemm: debug bounds check failed";
        default: return "unknown status";
    }
}

extern "C" int hgemm_sm100_read_status(int32_t* value, int clear) {
    if (value == nullptr) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    const DeviceInfo* dev = nullptr;
    int rc = device_info(&dev);
    if (rc != HGEMM_SM100_OK) return rc;
    if (cudaDeviceSynchronize() != cudaSuccess) return HGEMM_SM100_ERR_CUDA;
    int v = 0;
    if (cudaMemcpy(&v, dev->status_word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess)
        return HGEMM_SM100_ERR_CUDA;
    *value = v;
    if (clear && cudaMemset(dev->status_word, 0, sizeof(int)) != cudaSuccess) return HGEMM_SM100_ERR_CUDA;
    return HGEMM_SM100_OK;
}

// ============================================================ debug build ==

extern "C" int hgemm_sm100_debug_build(void) {
#ifdef HGEMM_DEBUG
    return 1;
#else
    return 0;
#endif
}

extern "C" int hgemm_sm100_debug_read(int32_t* line, int64_t* index0, int64_t* index1, int clear) {
    if (line == nullptr || index0 == nullptr || index1 == nullptr) return HGEMM_SM100_ERR_INVALID_ARGUMENT;
    *line = 0;
    *index0 = *index1 = 0;
#ifdef HGEMM_DEBUG
    const DeviceInfo* dev = nullptr;
    const int rc = device_info(&dev);
    if (rc != HGEMM_SM100_OK) return rc;
    if (cudaDeviceSynchronize() != cudaSuccess) return HGEMM_SM100_ERR_CUDA;
    DebugRecord rec{};
    if (cudaMemcpyFromSymbol(&rec, g_debug_record, sizeof(rec)) != cudaSuccess) return HGEMM_SM100_ERR_CUDA;
    *line = rec.line;
    *index0 = rec.index0;
    *index1 = rec.index1;
    if (clear) {
        const DebugRecord zero{};
        if (cudaMemcpyToSymbol(g_debug_record, &zero, sizeof(zero)) != cudaSuccess) return HGEMM_SM100_ERR_CUDA;
    }
#else
    (void)clear;
#endif
    return HGEMM_SM100_OK;
}

extern "C" int hgemm_sm100_debug_vec_touches(uint64_t vec, uint64_t base, int64_t rows, int64_t cols, int64_t ld,
                                             int32_t esize) {
    if (ld < cols || ld <= 0) return 0;
    return vec_touches_matrix(static_cast<uintptr_t>(vec), Extent{static_cast<uintptr_t>(base), rows, cols, ld, esize})
               ? 1 : 0;
}

extern "C" int hgemm_sm100_debug_span_in(uint64_t ptr, int64_t count, uint64_t base, int64_t rows, int64_t cols,
                                         int64_t ld, int32_t esize) {
    if (ld < cols || ld <= 0) return 0;
    return span_in_matrix(static_cast<uintptr_t>(ptr), count,
                          Extent{static_cast<uintptr_t>(base), rows, cols, ld, esize}) ? 1 : 0;
}

// ================================================ static-scratch entry point ==
//
// For callers that cannot allocate device memory at call time: the stream-K
// scratch is the file-scope array g_static_scratch (above) instead of a caller
// workspace; its device address on the current device comes from
// device_info(), which looks it up on the first call of any entry point on
// that device.

extern "C" int hgemm_sm100_run_static_scratch(const HgemmSm100Args* args, void* stream_ptr) {
    int rc = check_args(args);
    if (rc != HGEMM_SM100_OK) return rc;
    const DeviceInfo* dev = nullptr;
    rc = device_info(&dev);
    if (rc != HGEMM_SM100_OK) return rc;
    int devid = 0;
    if (cudaGetDevice(&devid) != cudaSuccess) return HGEMM_SM100_ERR_CUDA;
    if (!fp16_tma_ok(args->a, args->lda) || !fp16_tma_ok(args->b, args->ldb))
        return HGEMM_SM100_ERR_INVALID_ARGUMENT;

    const bool automatic = args->config == HGEMM_SM100_CFG_AUTO;
    int32_t cfg = args->config;
    if (automatic) cfg = args->m <= 128 ? HGEMM_SM100_CFG_STREAMK_SWAPAB : HGEMM_SM100_CFG_STREAMK_128x256;
    if (!is_streamk(cfg) || cfg == HGEMM_SM100_CFG_STREAMK_PAIR_256x256) return HGEMM_SM100_ERR_UNKNOWN_CONFIG;
    if (cfg == HGEMM_SM100_CFG_STREAMK_SWAPAB && args->m > 128) cfg = HGEMM_SM100_CFG_STREAMK_128x256;

    const StreamKPlan sp = plan_streamk(cfg, args->m, args->n, args->k, dev->sms);
    if (sp.bytes > HGEMM_SM100_STATIC_SCRATCH_BYTES) {
        // A split tail that does not fit: `auto` runs whole tiles with the
        // persistent kernel (no scratch); an explicit stream-K request fails.
        if (!automatic) return HGEMM_SM100_ERR_SCRATCH_LIMIT;
        return run_core(*args, HGEMM_SM100_CFG_PERSISTENT_128x256, 1, *dev, devid,
                        static_cast<cudaStream_t>(stream_ptr), nullptr, 0);
    }
    uint8_t* scratch = sp.bytes > 0 ? dev->static_scratch : nullptr;
    return run_core(*args, cfg, 1, *dev, devid, static_cast<cudaStream_t>(stream_ptr), scratch,
                    scratch != nullptr ? HGEMM_SM100_STATIC_SCRATCH_BYTES : 0);
}
