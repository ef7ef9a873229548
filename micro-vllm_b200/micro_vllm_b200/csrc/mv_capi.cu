// C ABI of libmvdecode.so: argument checks, split-KV planning, TMA tensor-map
// construction and kernel dispatch for paged decode attention and paged KV
// append. Declarations and the contract live in include/mvdecode.h.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <unordered_map>
#include <string>
#include <type_traits>
#include <utility>

#include "mvdecode.h"
#include "paged_append.cuh"
#include "paged_chunk_mma.cuh"
#include "paged_chunk_umma.cuh"
#include "paged_decode_merge.cuh"
#include "paged_decode_mma.cuh"
#include "paged_decode_simt.cuh"
#include "paged_decode_stream.cuh"
#include "rope.cuh"
#include "row_ops.cuh"

namespace {

thread_local std::string g_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list args;
    va_start(args, fmt);
    vsnprintf(buf, sizeof(buf), fmt, args);
    va_end(args);
    g_error = buf;
    return code;
}

int cuda_fail(cudaError_t err, const char* what) {
    return fail(MV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

// ------------------------------------------------------------ device facts

constexpr int kMaxDevices = 64;

struct DeviceInfo {
    int sms = 0;
    int smem_optin = 0;
};

DeviceInfo g_devices[kMaxDevices];
std::mutex g_device_mutex;

int device_info(DeviceInfo* info) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(MV_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_device_mutex);
    DeviceInfo& d = g_devices[dev];
    if (d.sms == 0) {
        err = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
        if (err == cudaSuccess)
            err = cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        if (err != cudaSuccess) {
            d.sms = 0;
            return cuda_fail(err, "cudaDeviceGetAttribute");
        }
    }
    *info = d;
    return MV_OK;
}

// Launch with programmatic stream serialization: the grid may start while the
// previous grid in the stream drains; the kernels wait (griddepcontrol.wait)
// before touching any input.
template <typename... Params, typename... Args>
cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Kernel attributes already set on a device (a cudaFuncSetAttribute per
// launch costs host time every call): kernel -> dynamic shared memory bytes
// allowed, and whether the largest carveout was requested.
struct KernelAttrs {
    size_t smem_bytes = 48 * 1024;
    bool carveout = false;
    int ctas_per_sm = -1;  // resident CTAs per SM at ctas_smem bytes (-1: not asked yet)
    size_t ctas_smem = 0;
};
std::mutex g_attr_mutex;
std::unordered_map<const void*, KernelAttrs> g_attrs[kMaxDevices];

template <typename Kernel>
int set_kernel_attrs(Kernel kernel, size_t bytes, bool carveout) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(MV_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    KernelAttrs& attrs = g_attrs[dev][reinterpret_cast<const void*>(kernel)];
    if (bytes > attrs.smem_bytes) {
        err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
        if (err != cudaSuccess) return cuda_fail(err, "cudaFuncSetAttribute");
        attrs.smem_bytes = bytes;
    }
    if (carveout && !attrs.carveout) {
        err = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                   static_cast<int>(cudaSharedmemCarveoutMaxShared));
        if (err != cudaSuccess) return cuda_fail(err, "cudaFuncSetAttribute");
        attrs.carveout = true;
    }
    return MV_OK;
}

// Resident CTAs per SM of a kernel launched with `threads` threads and `bytes`
// of dynamic shared memory on the current device (asked once per kernel, device
// and size).
template <typename Kernel>
int kernel_ctas_per_sm(Kernel kernel, int threads, size_t bytes, int* ctas) {
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) return fail(MV_ERR_UNSUPPORTED, "device index %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_attr_mutex);
    KernelAttrs& attrs = g_attrs[dev][reinterpret_cast<const void*>(kernel)];
    if (attrs.ctas_per_sm < 0 || attrs.ctas_smem != bytes) {
        int n = 0;
        err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, threads, bytes);
        if (err != cudaSuccess) return cuda_fail(err, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        attrs.ctas_per_sm = n;
        attrs.ctas_smem = bytes;
    }
    *ctas = attrs.ctas_per_sm;
    return MV_OK;
}

// Opt a kernel into `bytes` of dynamic shared memory on the current device.
template <typename Kernel>
int ensure_smem(Kernel kernel, size_t bytes) {
    if (bytes <= 48 * 1024) return MV_OK;
    return set_kernel_attrs(kernel, bytes, false);
}

// As ensure_smem, and prefer the largest shared-memory carveout: left to
// itself the driver may pick a carveout that holds fewer CTAs than the
// kernel's registers allow.
template <typename Kernel>
int ensure_smem_carveout(Kernel kernel, size_t bytes) {
    return set_kernel_attrs(kernel, bytes, true);
}

// ---------------------------------------------------------------- planning

// Split grid's graded schedule: splits after the second hold pages_per_split /
// MV_LATER_SPLIT_DIV pages (at least 16; 1: all splits after the first alike).
// Measured on B200 (Qwen2.5-7B geometry, batch 64; graph of 8 steps): 128/64/64
// pages 60.65 us, 128/64/32 60.44 us, 128/64/16 60.25 us; the batch-256 layer
// unchanged (589.7-590.0 us).
#ifndef MV_LATER_SPLIT_DIV
#define MV_LATER_SPLIT_DIV 4
#endif

// Split grid with the multi-wave (graded) plan: the CTAs of the first
// MV_PREWAIT_WAVES_X4 / 4 waves of resident CTAs, in dispatch order, prefetch
// their first MV_PREWAIT_PAGES pages per warp into L2 before waiting for the
// previous grid (0 pages: none). Measured on B200 (Qwen2.5-7B geometry, batch
// 64; graph of 8 steps): 59.87 us without, 56.63 us with 4 pages over two waves
// (2 pages 59.03, 3 pages 58.30, 5-6 pages 56.6-57.0; one wave 57.4); the
// batch-256 and long-context layers unchanged or 0.5% faster. Grids of one wave
// (small batches) lose 0.5-7% with it -- the previous kernel ends before the
// prefetch's dependent loads do -- so only the graded plan takes it.
#ifndef MV_PREWAIT_PAGES
#define MV_PREWAIT_PAGES 4
#endif
#ifndef MV_PREWAIT_WAVES_X4
#define MV_PREWAIT_WAVES_X4 8
#endif

// Tensor-core kernel shape: warps per CTA and TMA stages per warp by head_dim
// (overridable at build time for tuning sweeps).
#ifndef MV_MMA_WARPS
#define MV_MMA_WARPS 4
#endif
#ifndef MV_STAGES_D64
#define MV_STAGES_D64 6
#endif
#ifndef MV_STAGES_D128
#define MV_STAGES_D128 2
#endif
#ifndef MV_STAGES_D256
#define MV_STAGES_D256 2
#endif
constexpr int kMmaWarps = MV_MMA_WARPS;
// The wide split-grid shape for grids of about one CTA per SM: twice the warps,
// deeper rings (192 KiB of stages), so one CTA keeps as many pages in flight
// as three default CTAs. head_dim 256 has no wide shape (stages too large).
constexpr int kWideWarps = 8;
constexpr int kWideStagesD64 = 6;
constexpr int kWideStagesD128 = 3;
constexpr int kMaxPagesPerSplitWide = 32 * kWideWarps;
#ifndef MV_CLUSTER_PAGES
#define MV_CLUSTER_PAGES 64
#endif
constexpr int64_t kClusterPages = MV_CLUSTER_PAGES;  // pages per CTA the cluster kernel aims for
constexpr int kMaxPagesPerSplit = 32 * kMmaWarps;

struct Geometry {
    int32_t batch, q_heads, kv_heads, head_dim, block_size;
    int64_t max_context_len;
    int32_t dtype;
};

int check_geometry(const Geometry& g) {
    if (g.batch <= 0 || g.q_heads <= 0 || g.kv_heads <= 0 || g.head_dim <= 0 || g.block_size <= 0)
        return fail(MV_ERR_INVALID_ARGUMENT,
                    "batch, head counts, head dimension and block size must be positive");
    if (g.q_heads % g.kv_heads)
        return fail(MV_ERR_INVALID_ARGUMENT, "query head count must be divisible by KV head count");
    if (g.max_context_len < 0) return fail(MV_ERR_INVALID_ARGUMENT, "max_context_len must be nonnegative");
    if (g.dtype != MV_DTYPE_F32 && g.dtype != MV_DTYPE_F16 && g.dtype != MV_DTYPE_BF16)
        return fail(MV_ERR_INVALID_ARGUMENT, "dtype must be MV_DTYPE_F32, MV_DTYPE_F16 or MV_DTYPE_BF16");
    if (g.batch > 65535 || g.kv_heads > 65535)
        return fail(MV_ERR_UNSUPPORTED, "batch and KV head count are limited to 65535");
    return MV_OK;
}

struct Plan {
    int path;
    int pages_per_split;
    int max_splits;
    int first_pages; // split grid: pages of split 0 when longer than pages_per_split (split-major order), else 0
    int later_pages = 0; // split grid with first_pages: pages of splits 2.. (0: pages_per_split)
    int cluster;     // cluster kernel: CTAs per (sequence, KV head)
    int nt;          // mma n-tiles (8 query heads each)
    int ctas;        // persistent grid size
    int warps;       // persistent warps in the grid
    size_t workspace;
    size_t counter_bytes;  // zero-initialised arrival counters at the start of the workspace
    size_t part_o_bytes;
    size_t part_lse_bytes;
    bool fused_merge;
    bool wide;       // split grid in the wide shape (kWideWarps warps, deeper rings)
    bool chunk_umma; // chunk query tiles of 128 rows on tcgen05 (else 64 rows on mma.sync)
    bool cuda_core;  // split grid with CUDA-core math (MV_FLAG_CUDA_CORE_MATH)
};

// Where a plan may take the per-warp stream schedule: paged decode with one
// query row per sequence (not chunks, not contiguous caches).
enum class StreamUse { kNo, kAllowed };

bool mma_shape_ok(const Geometry& g) {
    const int group = g.q_heads / g.kv_heads;
    return (g.dtype == MV_DTYPE_BF16 || g.dtype == MV_DTYPE_F16) && g.block_size == 16 &&
           (g.head_dim == 64 || g.head_dim == 128 || g.head_dim == 256) && group <= 16;
}

size_t round256(size_t bytes) { return (bytes + 255) / 256 * 256; }

// Every non-empty workspace starts with this many bytes of arrival counters
// (one per sequence x KV head). No path writes anything else there, so once a
// workspace is zero-filled its counters stay zero between completed calls.
constexpr size_t kCounterRegion = 256 * 1024;
constexpr int64_t kMaxCounters = kCounterRegion / sizeof(unsigned);
static_assert(kMaxCounters == mv::kCounterRegionSlots, "device and host agree on the counter region");

// Persistent kernel: stages per warp for each head_dim (~96 KiB of stages per CTA
// so two CTAs share an SM; one at head_dim 256), and the batch its prefix array fits.
template <int D> struct PersistentStages {
    static constexpr int value = D == 64 ? MV_STAGES_D64 : (D == 128 ? MV_STAGES_D128 : MV_STAGES_D256);
};
constexpr int kPersistentMaxBatch = 1023;

template <typename T, int D, int NT>
auto persistent_kernel() {
    return mv::paged_decode_persistent_kernel<T, D, NT, kMmaWarps, PersistentStages<D>::value>;
}

template <int D>
constexpr int persistent_smem() {
    return mv::PersistentShape<D, kMmaWarps, PersistentStages<D>::value>::smem_bytes(kPersistentMaxBatch);
}

// Resident CTAs per SM of the persistent kernel instance, cached per device.
template <typename T, int D, int NT>
int persistent_occupancy(int device, int* ctas_per_sm) {
    static int cache[kMaxDevices] = {0};
    static std::mutex mutex;
    std::lock_guard<std::mutex> lock(mutex);
    if (cache[device] == 0) {
        auto kernel = persistent_kernel<T, D, NT>();
        int rc = ensure_smem(kernel, persistent_smem<D>());
        if (rc != MV_OK) return rc;
        int blocks = 0;
        cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, kMmaWarps * 32,
                                                                        persistent_smem<D>());
        if (err != cudaSuccess) return cuda_fail(err, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        if (blocks < 1) return fail(MV_ERR_UNSUPPORTED, "persistent decode kernel does not fit an SM");
        cache[device] = blocks;
    }
    *ctas_per_sm = cache[device];
    return MV_OK;
}

template <typename T>
int persistent_occupancy_dispatch(int device, int dim, int nt, int* ctas_per_sm) {
    switch (dim * 4 + nt) {
        case 64 * 4 + 1: return persistent_occupancy<T, 64, 1>(device, ctas_per_sm);
        case 64 * 4 + 2: return persistent_occupancy<T, 64, 2>(device, ctas_per_sm);
        case 128 * 4 + 1: return persistent_occupancy<T, 128, 1>(device, ctas_per_sm);
        case 128 * 4 + 2: return persistent_occupancy<T, 128, 2>(device, ctas_per_sm);
        case 256 * 4 + 1: return persistent_occupancy<T, 256, 1>(device, ctas_per_sm);
        case 256 * 4 + 2: return persistent_occupancy<T, 256, 2>(device, ctas_per_sm);
        default: return fail(MV_ERR_UNSUPPORTED, "no tensor-core kernel for head_dim %d", dim);
    }
}

// Shared memory of the split-grid kernel's TMA stages (reused for the fused merge).
size_t grid_stage_bytes(int dim, bool wide) {
    const int stages = wide ? (dim == 64 ? kWideStagesD64 : kWideStagesD128)
                            : (dim == 64 ? MV_STAGES_D64 : (dim == 128 ? MV_STAGES_D128 : MV_STAGES_D256));
    return static_cast<size_t>(wide ? kWideWarps : kMmaWarps) * stages * 2 * (16 * static_cast<size_t>(dim) * 2);
}

// The per-warp stream schedule (paged_decode_stream_kernel), on request
// (MV_FLAG_STREAM): items of 8..64 pages, about four per warp. Measured on
// B200 it loses to the split grid (Qwen2.5-7B geometry, batch 64: 68.7 us per
// step with 32-page items, 77.6 us with 8-page ones, against 61.5 us; Qwen2.5-72B
// geometry, batch 256: 620-635 against 598 us): a warp streams only its own
// two stages, so items must be small for the queue to balance, and every item
// switch costs the warp ~2 us (claim, page IDs, q) that its ring cannot hide.
bool stream_plan(const Geometry& g, int32_t pages_per_split, uint32_t flags, const DeviceInfo& dev, Plan* plan) {
    if (!(flags & MV_FLAG_STREAM)) return false;
    const int64_t max_pages = (g.max_context_len + g.block_size - 1) / g.block_size;
    const bool shape = plan->path == MV_PATH_TMA_MMA && !plan->wide && !plan->cuda_core && plan->nt == 1 &&
                       (g.head_dim == 64 || g.head_dim == 128) && g.batch <= mv::kStreamMaxBatch &&
                       g.max_context_len < (int64_t(1) << 30) &&
                       !(flags & (MV_FLAG_FUSED_MERGE | MV_FLAG_CLUSTER | MV_FLAG_PERSISTENT | MV_FLAG_WIDE |
                                  MV_FLAG_CUDA_CORE_MATH | MV_FLAG_SPLIT_GRID));
    if (!shape) return false;
    const int64_t warps = static_cast<int64_t>(dev.sms) * mv::kStreamWarps;
    const int64_t est_pages = static_cast<int64_t>(g.batch) * g.kv_heads * std::max<int64_t>(max_pages, 1) / 2;
    int64_t items = pages_per_split;
    if (items == 0) {
        // About four items per warp, and at most 32 per segment (one round of
        // loads in the warp merge; partials bounded by 32 rows per query row).
        const int64_t want = est_pages / (4 * warps);
        items = 8;
        while ((items * 2 <= want || items * 32 < max_pages) && items < mv::kStreamMaxItemPages) items *= 2;
    }
    if (items < 1 || items > mv::kStreamMaxItemPages) return false;
    const int64_t splits = std::max<int64_t>(1, (max_pages + items - 1) / items);
    if (splits > 8192) return false;
    plan->path = MV_PATH_TMA_MMA_STREAM;
    plan->pages_per_split = static_cast<int>(items);
    plan->first_pages = 0;
    plan->max_splits = static_cast<int>(splits);
    plan->ctas = dev.sms;
    plan->warps = dev.sms * mv::kStreamWarps;
    plan->fused_merge = false;
    plan->counter_bytes = kCounterRegion;  // the item queue's counters
    plan->part_o_bytes = plan->part_lse_bytes = 0;
    if (splits > 1) {
        const size_t rows = static_cast<size_t>(g.batch) * g.q_heads * splits;
        plan->part_o_bytes = round256(rows * g.head_dim * sizeof(float));
        plan->part_lse_bytes = round256(rows * sizeof(float));
    }
    plan->workspace = plan->counter_bytes + plan->part_o_bytes + plan->part_lse_bytes;
    return true;
}

int make_plan(const Geometry& g, int32_t pages_per_split, uint32_t flags, bool aligned_for_tma,
              Plan* plan, StreamUse stream_use = StreamUse::kNo) {
    int rc = check_geometry(g);
    if (rc != MV_OK) return rc;
    DeviceInfo dev;
    rc = device_info(&dev);
    if (rc != MV_OK) return rc;
    int device = 0;
    cudaGetDevice(&device);
    const int group = g.q_heads / g.kv_heads;
    if (pages_per_split < 0) return fail(MV_ERR_INVALID_ARGUMENT, "pages_per_split must be nonnegative");
    const bool mma = !(flags & MV_FLAG_FORCE_SIMT) && aligned_for_tma && mma_shape_ok(g);
    const bool persistent = mma && pages_per_split == 0 && (flags & MV_FLAG_PERSISTENT) &&
                            g.batch <= kPersistentMaxBatch &&
                            static_cast<int64_t>(g.batch) * g.kv_heads < (int64_t(1) << 31);
    plan->path = persistent ? MV_PATH_TMA_MMA_PERSISTENT : (mma ? MV_PATH_TMA_MMA : MV_PATH_SIMT);
    plan->nt = group <= 8 ? 1 : 2;
    plan->ctas = plan->warps = 0;
    plan->cluster = 0;
    plan->counter_bytes = plan->part_o_bytes = plan->part_lse_bytes = 0;
    plan->fused_merge = false;
    plan->wide = false;
    plan->chunk_umma = false;
    plan->first_pages = 0;
    plan->later_pages = 0;
    plan->cuda_core = false;
    const int64_t max_pages = (g.max_context_len + g.block_size - 1) / g.block_size;

    // Opt-in: sequences up to kClusterPages x 8 pages split over a cluster of up
    // to 8 CTAs of <= kClusterPages pages each, combined through distributed
    // shared memory -- no partials in HBM, no merge pass. Measured on B200 it
    // loses to the split grid (a cluster's CTAs wait for its slowest one).
    if (mma && !persistent && pages_per_split == 0 && (flags & MV_FLAG_CLUSTER) &&
        max_pages <= 8 * kClusterPages) {
        int csize = 1;
        while (csize * kClusterPages < max_pages) csize *= 2;
        plan->path = MV_PATH_TMA_MMA_CLUSTER;
        plan->cluster = csize;
        plan->pages_per_split = static_cast<int>((max_pages + csize - 1) / csize);
        plan->max_splits = 1;
        plan->workspace = 0;
        return MV_OK;
    }

    if (persistent) {
        int per_sm = 0;
        rc = g.dtype == MV_DTYPE_BF16 ? persistent_occupancy_dispatch<__nv_bfloat16>(device, g.head_dim, plan->nt, &per_sm)
                                      : persistent_occupancy_dispatch<__half>(device, g.head_dim, plan->nt, &per_sm);
        if (rc != MV_OK) return rc;
        plan->ctas = dev.sms * per_sm;
        plan->warps = plan->ctas * kMmaWarps;
        plan->pages_per_split = 0;
        plan->max_splits = 1;
        const size_t rows = static_cast<size_t>(plan->warps) * 2 * 8 * plan->nt;  // 2 partial slots per warp
        plan->part_o_bytes = round256(rows * g.head_dim * sizeof(float));
        plan->part_lse_bytes = round256(rows * sizeof(float));
        plan->counter_bytes = kCounterRegion;
        plan->workspace = plan->counter_bytes + plan->part_o_bytes + plan->part_lse_bytes +
                          round256((static_cast<size_t>(g.batch) + 1) * sizeof(int64_t));
        return MV_OK;
    }

    // The wide shape (8 warps, deeper rings, about one CTA per SM) when the
    // batch has few (sequence, KV head) segments with up to 1024 pages each:
    // measured on B200 it wins there (e.g. 32 x 2 segments of ~40 pages: 9.8 vs
    // 12.7 us; 4 x 8 of 1024: 51 vs 56 us) and loses with many segments (the
    // default grid packs three CTAs per SM) or very few (more, smaller CTAs win).
    const int64_t segments = static_cast<int64_t>(g.batch) * g.kv_heads;
    const bool auto_wide = pages_per_split == 0 && !(flags & (MV_FLAG_FUSED_MERGE | MV_FLAG_CLUSTER | MV_FLAG_STREAM)) &&
                           segments >= 16 && segments <= dev.sms / 2 && max_pages <= 1024;
    plan->wide = plan->path == MV_PATH_TMA_MMA && ((flags & MV_FLAG_WIDE) || auto_wide) && g.head_dim != 256;
    // The CUDA-core variant runs the default shape only (it is a comparison point).
    plan->cuda_core = plan->path == MV_PATH_TMA_MMA && (flags & MV_FLAG_CUDA_CORE_MATH) && group <= 8 &&
                      (g.head_dim == 64 || g.head_dim == 128);
    if (plan->cuda_core) plan->wide = false;
    const int64_t max_pps = plan->wide ? kMaxPagesPerSplitWide : kMaxPagesPerSplit;
    int64_t pps = pages_per_split;
    if (pps == 0 && plan->wide) {
        // One split when a sequence fits 64 pages (no merge pass); otherwise
        // about one wide CTA per SM: each segment's pages over SMs / segments
        // splits, in multiples of 32 pages (32..256).
        if (max_pages <= 64) {
            pps = std::max<int64_t>(1, max_pages);
        } else {
            const int64_t per_segment = std::max<int64_t>(1, dev.sms / std::max<int64_t>(segments, 1));
            pps = (max_pages + per_segment - 1) / per_segment;
            pps = std::min<int64_t>(std::max<int64_t>((pps + 31) / 32 * 32, 32), kMaxPagesPerSplitWide);
        }
    }
    const bool auto_pps = pps == 0;
    if (pps == 0) {
        // Splits of 16..128 pages (tensor cores), sized so the batch's pages -- estimated as half
        // the max_context_len bound per sequence -- fill about one wave of
        // resident CTAs (three per SM). Measured on B200: longer splits lose to
        // the tail of the last wave, shorter ones to per-CTA start-up and the
        // merge; 64 pages at batch 64 x 4 KV heads x ~2.5k tokens, 128 at long
        // contexts.
        const int64_t pages = static_cast<int64_t>(g.batch) * g.kv_heads * std::max<int64_t>(max_pages, 1) / 2;
        const int64_t target = static_cast<int64_t>(dev.sms) * 3;
        const int64_t want = (pages + target - 1) / target;
        // The CUDA-core kernel walks 32-token tiles one after another, so small
        // batches want splits down to one tile each (more CTAs, shorter chains).
        pps = plan->path == MV_PATH_SIMT ? std::max<int64_t>(1, (mv::kSimtTile + g.block_size - 1) / g.block_size)
                                         : 16;
        while (pps * 2 <= want && pps < kMaxPagesPerSplit) pps *= 2;
        // Tensor cores: at most 64 splits per sequence. Measured on B200 (Qwen3-8B
        // geometry, one KV head of 8 sequences of 32k-131k tokens -- a rank's
        // shard at 8 GPUs): 64-page splits (126 per sequence) 71.9 us, 128-page
        // ones 63.8 us -- half the CTAs, and half the pieces for the merge.
        if (plan->path == MV_PATH_TMA_MMA)
            while (pps * 64 < max_pages && pps < kMaxPagesPerSplit) pps *= 2;
        pps = std::min<int64_t>(pps, kMaxPagesPerSplit);
    }
    if (plan->path == MV_PATH_TMA_MMA && pps > max_pps)
        return fail(MV_ERR_INVALID_ARGUMENT, "pages_per_split above %d for the tensor-core kernel",
                    static_cast<int>(max_pps));
    // The automatic plan of the (default-shape) tensor-core split grid makes
    // each sequence's first split twice as long (up to kMaxPagesPerSplit pages)
    // and dispatches the grid split-major: every first split starts in the
    // first wave, the shorter later splits fill the tail, and sequences of up
    // to 2 x pps pages need no merge. Measured on B200 (Qwen2.5-7B geometry,
    // batch 64, 1k-4k tokens): 62.1 us per step against 65.0 us with uniform
    // 64-page splits and 62.8 us with uniform 128-page splits.
    // Splits after the second are shorter again (MV_LATER_SPLIT_DIV), so the
    // CTAs dispatched last are the smallest. Re-measured with the first wave's
    // L2 warm-up (MV_PREWAIT_PAGES): first splits of 96 / 112 / 128 / 160 / 192 / 256
    // pages 62.0 / 59.7 / 56.9 / 62.5 / 66.6 / 74.4 us; later splits of 16 /
    // 32 / 64 pages 56.9 / 57.1 / 57.8 us.
    // Only where the grid is more than one wave: with every CTA resident at
    // once the longest split sets the time (batch 1 x 4096 tokens: 13.8 us
    // with a 32-page first split, 10.3 us without).
    if (auto_pps && plan->path == MV_PATH_TMA_MMA && !plan->wide) {
        const int64_t first = std::min<int64_t>(2 * pps, kMaxPagesPerSplit);
        const int64_t est_ctas = static_cast<int64_t>(g.batch) * g.kv_heads *
                                 ((std::max<int64_t>(max_pages, 1) / 2 + pps - 1) / pps);
        if (first > pps && est_ctas > static_cast<int64_t>(dev.sms) * 3) {
            plan->first_pages = static_cast<int>(first);
            // Graded only while the plan stays at 8 splits or fewer: long contexts
            // would otherwise get dozens of small splits (more CTAs, partials and
            // merge work for no gain).
            const int64_t later = std::max<int64_t>(16, pps / MV_LATER_SPLIT_DIV);
            const int64_t graded = max_pages <= first + pps ? 2 : 2 + (max_pages - first - pps + later - 1) / later;
            if (MV_LATER_SPLIT_DIV > 1 && later < pps && graded <= 8) plan->later_pages = static_cast<int>(later);
        }
    }
    const int64_t first = plan->first_pages;
    const int64_t later = plan->later_pages > 0 ? plan->later_pages : pps;
    const int64_t splits = first > 0 ? (max_pages <= first ? 1 : max_pages <= first + pps ? 2
                                                               : 2 + (max_pages - first - pps + later - 1) / later)
                                     : std::max<int64_t>(1, (max_pages + pps - 1) / pps);
    if (splits > 8192) return fail(MV_ERR_UNSUPPORTED, "more than 8192 splits: raise pages_per_split");
    plan->pages_per_split = static_cast<int>(pps);
    plan->max_splits = static_cast<int>(splits);
    if (splits > 1) {
        const size_t rows = static_cast<size_t>(g.batch) * g.q_heads * splits;
        plan->part_o_bytes = round256(rows * g.head_dim * sizeof(float));
        plan->part_lse_bytes = round256(rows * sizeof(float));
        // The tensor-core split grid merges in its last CTA per segment when the
        // segment's G x splits weights fit the CTA's stage memory.
        // Merging in the last split CTA of each segment holds that CTA's SM slot
        // through a latency-bound merge; measured on B200 it cost more than the
        // separate merge pass (launched early with PDL), so it is opt-in.
        plan->fused_merge = (flags & MV_FLAG_FUSED_MERGE) && plan->path == MV_PATH_TMA_MMA &&
                            static_cast<size_t>(group) * splits * sizeof(float) <= grid_stage_bytes(g.head_dim, plan->wide) &&
                            static_cast<int64_t>(g.batch) * g.kv_heads <= kMaxCounters - mv::kStreamCounterSlots;
        plan->counter_bytes = kCounterRegion;
    }
    plan->workspace = plan->counter_bytes + plan->part_o_bytes + plan->part_lse_bytes;
    if (stream_use == StreamUse::kAllowed && stream_plan(g, pages_per_split, flags, dev, plan)) return MV_OK;
    if ((flags & MV_FLAG_STREAM) && stream_use == StreamUse::kAllowed)
        return fail(MV_ERR_UNSUPPORTED,
                    "MV_FLAG_STREAM needs the tensor-core kernel (bf16/fp16, page 16, head_dim 64/128, GQA "
                    "group <= 8, TMA-aligned caches), at most %d sequences, pages_per_split <= %d and no other "
                    "schedule flag", mv::kStreamMaxBatch, mv::kStreamMaxItemPages);
    if (plan->path == MV_PATH_SIMT) {
        const size_t smem = mv::simt_smem_bytes(group, g.head_dim);
        if (smem > static_cast<size_t>(dev.smem_optin))
            return fail(MV_ERR_UNSUPPORTED,
                        "GQA group %d x head_dim %d needs %zu bytes of shared memory (device limit %d)",
                        group, g.head_dim, smem, dev.smem_optin);
    }
    return MV_OK;
}

// Plan of a chunk of `tokens` query tokens per sequence; g.batch counts query
// rows (sequences x tokens). Where query tiles apply -- the split grid's
// tensor-core plan, head_dim 64/128 and at least 16 rows (token x query head)
// per (sequence, KV head) -- the chunk runs as tiles of 128 rows on tcgen05
// (at least kUmmaMinRows rows, unless MV_FLAG_CHUNK_MMA_SYNC) or of 64 rows on
// mma.sync, and its splits are sized for those tiles: enough equal splits of
// the max_context_len bound for at most one wave (tcgen05, rounded down) or two waves
// (mma.sync) of resident tile CTAs, none shorter than kChunkMinPages pages. The plan is the split grid's either way,
// so a call whose query is not aligned for a tile kernel runs the next kernel
// down (tcgen05 -> mma.sync tiles -> row per token) on the same splits.
constexpr int64_t kChunkCtasPerSm = 3;
constexpr int64_t kUmmaCtasPerSm = 2;
constexpr int64_t kUmmaMinRows = 64;
constexpr int64_t kChunkMinPages = 32;

int make_chunk_plan(const Geometry& g, int32_t tokens, int32_t pages_per_split, uint32_t flags,
                    bool aligned_for_tma, Plan* plan, bool* tiles) {
    int rc = make_plan(g, pages_per_split, flags, aligned_for_tma, plan);
    if (rc != MV_OK) return rc;
    const int group = g.q_heads / g.kv_heads;
    *tiles = !(flags & MV_FLAG_CHUNK_ROWS) && plan->path == MV_PATH_TMA_MMA &&
             (g.head_dim == 64 || g.head_dim == 128) && static_cast<int64_t>(tokens) * group >= 16 &&
             pages_per_split <= mv::kChunkMaxPages;
    if (!*tiles) return MV_OK;
    DeviceInfo dev;
    rc = device_info(&dev);
    if (rc != MV_OK) return rc;
    plan->chunk_umma = !(flags & MV_FLAG_CHUNK_MMA_SYNC) && static_cast<int64_t>(tokens) * group >= kUmmaMinRows;
    const int64_t tile_rows = plan->chunk_umma ? mv::kUmmaRows : mv::kChunkRows;
    const int64_t max_pages = std::max<int64_t>(1, (g.max_context_len + 15) / 16);
    int64_t pps = pages_per_split;
    if (pps == 0) {
        const int64_t sequences = g.batch / tokens;
        const int64_t q_tiles = (static_cast<int64_t>(tokens) * group + tile_rows - 1) / tile_rows;
        const int64_t tiles_total = sequences * g.kv_heads * q_tiles;
        // tcgen05 tiles: at most one wave of resident CTAs, rounding the split
        // count down -- every split adds a partial row per query row (written,
        // then read by the merge: 4 sequences x 256 tokens x 12 heads x 3
        // splits is 19 MB against 5 MB of K/V), so splitting pays only while
        // the tiles leave much of the GPU idle. Measured on B200 (graph of
        // back-to-back calls): 96 tiles: 3 splits 33.1 us, 1 split 40.2 us;
        // 192 tiles: 1 split 63.1 / 40.5 us against 2 splits 84.1 / 64.0 us.
        // mma.sync tiles: two waves.
        const int64_t target = static_cast<int64_t>(dev.sms) * (plan->chunk_umma ? kUmmaCtasPerSm : kChunkCtasPerSm * 2);
        int64_t splits = plan->chunk_umma ? std::max<int64_t>(1, target / tiles_total)
                                          : std::max<int64_t>(1, (target + tiles_total - 1) / tiles_total);
        splits = std::min<int64_t>(splits, std::max<int64_t>(1, (max_pages + kChunkMinPages - 1) / kChunkMinPages));
        pps = std::min<int64_t>((max_pages + splits - 1) / splits, mv::kChunkMaxPages);
    }
    const int64_t splits = std::max<int64_t>(1, (max_pages + pps - 1) / pps);
    if (splits > 8192) return fail(MV_ERR_UNSUPPORTED, "more than 8192 splits: raise pages_per_split");
    plan->wide = false;
    plan->fused_merge = false;
    plan->first_pages = 0;
    plan->pages_per_split = static_cast<int>(pps);
    plan->max_splits = static_cast<int>(splits);
    plan->counter_bytes = plan->part_o_bytes = plan->part_lse_bytes = 0;
    if (splits > 1) {
        const size_t rows = static_cast<size_t>(g.batch) * g.q_heads * splits;
        plan->part_o_bytes = round256(rows * g.head_dim * sizeof(float));
        plan->part_lse_bytes = round256(rows * sizeof(float));
        plan->counter_bytes = kCounterRegion;
    }
    plan->workspace = plan->counter_bytes + plan->part_o_bytes + plan->part_lse_bytes;
    return MV_OK;
}

bool tma_aligned(const void* k_cache, const void* v_cache) {
    return (reinterpret_cast<uintptr_t>(k_cache) % 16 == 0) && (reinterpret_cast<uintptr_t>(v_cache) % 16 == 0);
}

// ------------------------------------------------------------ tensor maps

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult status;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &status) ==
                cudaSuccess &&
            status == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

struct MapKey {
    const void* base;
    int32_t kind;          // 0: page pool, 1: contiguous cache, 2: page pool in 64-dim boxes
    int32_t dim, dtype;
    int64_t extent[3];     // pool: (pages, heads, 0); contiguous: (tokens, heads, sequences)
    int64_t stride[3];     // contiguous: element strides (token, head, sequence)
    bool operator==(const MapKey& o) const {
        return base == o.base && kind == o.kind && dim == o.dim && dtype == o.dtype &&
               extent[0] == o.extent[0] && extent[1] == o.extent[1] && extent[2] == o.extent[2] &&
               stride[0] == o.stride[0] && stride[1] == o.stride[1] && stride[2] == o.stride[2];
    }
};

struct MapEntry {
    MapKey key;
    CUtensorMap map;
    bool used;
};

constexpr int kMapCache = 64;
MapEntry g_maps[kMapCache];
int g_map_next = 0;
std::mutex g_map_mutex;

// Page pool [num_blocks, heads, 16, dim] viewed as 5-D (d % 64, slot, d / 64,
// head, page) so one box = one page of one head, stored as dim/64 swizzled
// [16 x 128 B] sub-tiles.
int cached_tensor_map(const MapKey& key, CUtensorMap* out);

int page_tensor_map(const void* base, int64_t num_blocks, int heads, int dim, int dtype, CUtensorMap* out) {
    const MapKey key{base, 0, dim, dtype, {num_blocks, heads, 0}, {0, 0, 0}};
    return cached_tensor_map(key, out);
}

// The same pool with one 64-dim half of a page (16 rows of 128 B) per box, so
// a page's halves can land in separate places.
int page_half_tensor_map(const void* base, int64_t num_blocks, int heads, int dim, int dtype, CUtensorMap* out) {
    const MapKey key{base, 2, dim, dtype, {num_blocks, heads, 0}, {0, 0, 0}};
    return cached_tensor_map(key, out);
}

// Contiguous cache [sequences, heads, tokens, dim] with element strides, viewed
// as 5-D (d % 64, token, d / 64, head, sequence): one box = 16 tokens of one
// head, the same shared-memory tile as a page; tokens past the cache read as 0.
int contiguous_tensor_map(const void* base, int64_t tokens, int heads, int64_t sequences, int dim,
                          const int64_t* strides, int dtype, CUtensorMap* out) {
    const MapKey key{base, 1, dim, dtype, {tokens, heads, sequences}, {strides[0], strides[1], strides[2]}};
    return cached_tensor_map(key, out);
}

int cached_tensor_map(const MapKey& key, CUtensorMap* out) {
    std::lock_guard<std::mutex> lock(g_map_mutex);
    for (int i = 0; i < kMapCache; ++i) {
        if (g_maps[i].used && g_maps[i].key == key) {
            *out = g_maps[i].map;
            return MV_OK;
        }
    }
    auto encode = encode_fn();
    if (!encode) return fail(MV_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable from the driver");
    const int dim = key.dim;
    const cuuint64_t row = static_cast<cuuint64_t>(dim) * 2;
    cuuint64_t dims[5];
    cuuint64_t strides[4];
    if (key.kind == 0 || key.kind == 2) {
        const cuuint64_t heads = static_cast<cuuint64_t>(key.extent[1]);
        const cuuint64_t d5[5] = {64, 16, static_cast<cuuint64_t>(dim / 64), heads,
                                  static_cast<cuuint64_t>(key.extent[0])};
        const cuuint64_t s4[4] = {row, 128, 16 * row, heads * 16 * row};
        std::memcpy(dims, d5, sizeof(dims));
        std::memcpy(strides, s4, sizeof(strides));
    } else {
        const cuuint64_t d5[5] = {64, static_cast<cuuint64_t>(key.extent[0]), static_cast<cuuint64_t>(dim / 64),
                                  static_cast<cuuint64_t>(key.extent[1]), static_cast<cuuint64_t>(key.extent[2])};
        const cuuint64_t s4[4] = {static_cast<cuuint64_t>(key.stride[0]) * 2, 128,
                                  static_cast<cuuint64_t>(key.stride[1]) * 2, static_cast<cuuint64_t>(key.stride[2]) * 2};
        std::memcpy(dims, d5, sizeof(dims));
        std::memcpy(strides, s4, sizeof(strides));
    }
    cuuint32_t box[5] = {64, 16, key.kind == 2 ? 1u : static_cast<cuuint32_t>(dim / 64), 1, 1};
    cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
    CUtensorMap map;
    CUresult r = encode(&map, key.dtype == MV_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                        5, const_cast<void*>(key.base), dims, strides, box, elem_strides,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MV_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
    g_maps[g_map_next] = MapEntry{key, map, true};
    g_map_next = (g_map_next + 1) % kMapCache;
    *out = map;
    return MV_OK;
}

// ----------------------------------------------------------------- launch

template <typename T, int D, int NT, int WARPS, int STAGES, bool FMA = false>
int launch_mma_shape(const mv::DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, dim3 grid,
                     cudaStream_t stream) {
    using Shape = mv::MmaDecodeShape<D, NT, WARPS, STAGES>;
    auto kernel = mv::paged_decode_mma_kernel<T, D, NT, WARPS, STAGES, FMA>;
    constexpr int smem = Shape::kSmemBytes + (FMA ? mv::fma_extra_smem<T, D, WARPS>() : 0);
    int rc = ensure_smem(kernel, smem);
    if (rc != MV_OK) return rc;
    mv::DecodeParams q = p;
    if (MV_PREWAIT_PAGES > 0 && p.first_pages > 0 && !p.contiguous && p.context_lens && p.q_tokens == 1) {
        int per_sm = 0;
        DeviceInfo dev;
        rc = kernel_ctas_per_sm(kernel, WARPS * 32, smem, &per_sm);
        if (rc == MV_OK) rc = device_info(&dev);
        if (rc != MV_OK) return rc;
        q.prewait_ctas = dev.sms * per_sm * MV_PREWAIT_WAVES_X4 / 4;
        q.prewait_pages = MV_PREWAIT_PAGES;
    }
    cudaError_t err = launch_pdl(kernel, grid, dim3(WARPS * 32), smem, stream, q, kmap, vmap);
    return err == cudaSuccess ? MV_OK : cuda_fail(err, "decode kernel launch");
}

template <typename T, int D, int NT>
int launch_mma(const mv::DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, dim3 grid,
               bool wide, bool cuda_core, cudaStream_t stream) {
    constexpr int STAGES = D == 64 ? MV_STAGES_D64 : (D == 128 ? MV_STAGES_D128 : MV_STAGES_D256);
    if constexpr (NT == 1 && D != 256) {
        if (cuda_core) return launch_mma_shape<T, D, 1, kMmaWarps, STAGES, true>(p, kmap, vmap, grid, stream);
    }
    if constexpr (D != 256) {
        constexpr int WIDE_STAGES = D == 64 ? kWideStagesD64 : kWideStagesD128;
        if (wide) return launch_mma_shape<T, D, NT, kWideWarps, WIDE_STAGES>(p, kmap, vmap, grid, stream);
    }
    return launch_mma_shape<T, D, NT, kMmaWarps, STAGES>(p, kmap, vmap, grid, stream);
}

template <typename T>
int launch_mma_dispatch(const mv::DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                        dim3 grid, int nt, bool wide, bool cuda_core, cudaStream_t stream) {
    switch (p.head_dim * 4 + nt) {
        case 64 * 4 + 1: return launch_mma<T, 64, 1>(p, kmap, vmap, grid, wide, cuda_core, stream);
        case 64 * 4 + 2: return launch_mma<T, 64, 2>(p, kmap, vmap, grid, wide, cuda_core, stream);
        case 128 * 4 + 1: return launch_mma<T, 128, 1>(p, kmap, vmap, grid, wide, cuda_core, stream);
        case 128 * 4 + 2: return launch_mma<T, 128, 2>(p, kmap, vmap, grid, wide, cuda_core, stream);
        case 256 * 4 + 1: return launch_mma<T, 256, 1>(p, kmap, vmap, grid, wide, cuda_core, stream);
        case 256 * 4 + 2: return launch_mma<T, 256, 2>(p, kmap, vmap, grid, wide, cuda_core, stream);
        default: return fail(MV_ERR_UNSUPPORTED, "no tensor-core kernel for head_dim %d", p.head_dim);
    }
}

// One CTA per output row (query head, sequence).
dim3 merge_grid(const mv::DecodeParams& p) { return dim3(p.q_heads, p.batch); }

// The split grid's merge pass: a warp per output row where head_dim <= 128 is a
// multiple of 4 and rows have at most 32 pieces; a CTA per row whose warps
// share the pieces for up to 128; else a CTA per row looping over them.
template <typename T>
cudaError_t launch_split_merge(const mv::DecodeParams& p, cudaStream_t stream) {
    const bool columns = p.head_dim % 4 == 0 && p.head_dim <= 128;
    if (columns && p.max_splits <= 32) {
        const int64_t rows = static_cast<int64_t>(p.batch) * p.q_heads;
        const dim3 grid(static_cast<unsigned>((rows + mv::kWarpMergeRows - 1) / mv::kWarpMergeRows));
        return launch_pdl(mv::paged_decode_merge_warp_kernel<T>, grid, dim3(mv::kWarpMergeRows * 32), 0, stream, p);
    }
    if (columns && p.max_splits <= mv::kManyMergeMax)
        return launch_pdl(mv::paged_decode_merge_many_kernel<T>, merge_grid(p), dim3(mv::kManyMergeWarps * 32), 0,
                          stream, p);
    return launch_pdl(mv::paged_decode_merge_kernel<T>, merge_grid(p), dim3(mv::kMergeThreads), 0, stream, p);
}

template <typename T, int D, int NT>
int launch_persistent(const mv::DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      int ctas, cudaStream_t stream) {
    auto kernel = persistent_kernel<T, D, NT>();
    int rc = ensure_smem(kernel, persistent_smem<D>());
    if (rc != MV_OK) return rc;
    cudaError_t err = launch_pdl(kernel, dim3(ctas), dim3(kMmaWarps * 32), persistent_smem<D>(), stream,
                                 p, kmap, vmap);
    if (err != cudaSuccess) return cuda_fail(err, "persistent decode kernel launch");
    err = launch_pdl(mv::paged_decode_persistent_merge_kernel<T, 8 * NT>, merge_grid(p),
                     dim3(mv::kMergeThreads), 0, stream, p);
    return err == cudaSuccess ? MV_OK : cuda_fail(err, "merge kernel launch");
}

// The per-warp stream schedule: one CTA per SM.
template <typename T, int D>
int launch_stream(const mv::DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap, int ctas,
                  cudaStream_t stream) {
    auto kernel = mv::paged_decode_stream_kernel<T, D>;
    int rc = ensure_smem(kernel, mv::StreamShape<D>::kSmemBytes);
    if (rc != MV_OK) return rc;
    cudaError_t err = launch_pdl(kernel, dim3(ctas), dim3(mv::kStreamWarps * 32), mv::StreamShape<D>::kSmemBytes,
                                 stream, p, kmap, vmap);
    return err == cudaSuccess ? MV_OK : cuda_fail(err, "stream decode kernel launch");
}

template <typename T>
int launch_persistent_dispatch(const mv::DecodeParams& p, const CUtensorMap& kmap,
                               const CUtensorMap& vmap, int ctas, int nt, cudaStream_t stream) {
    switch (p.head_dim * 4 + nt) {
        case 64 * 4 + 1: return launch_persistent<T, 64, 1>(p, kmap, vmap, ctas, stream);
        case 64 * 4 + 2: return launch_persistent<T, 64, 2>(p, kmap, vmap, ctas, stream);
        case 128 * 4 + 1: return launch_persistent<T, 128, 1>(p, kmap, vmap, ctas, stream);
        case 128 * 4 + 2: return launch_persistent<T, 128, 2>(p, kmap, vmap, ctas, stream);
        case 256 * 4 + 1: return launch_persistent<T, 256, 1>(p, kmap, vmap, ctas, stream);
        case 256 * 4 + 2: return launch_persistent<T, 256, 2>(p, kmap, vmap, ctas, stream);
        default: return fail(MV_ERR_UNSUPPORTED, "no tensor-core kernel for head_dim %d", p.head_dim);
    }
}

template <typename T, int D, int NT>
int launch_cluster(const mv::DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                   int csize, cudaStream_t stream) {
    constexpr int STAGES = D == 64 ? MV_STAGES_D64 : (D == 128 ? MV_STAGES_D128 : MV_STAGES_D256);
    using Shape = mv::ClusterShape<D, NT, kMmaWarps, STAGES>;
    auto kernel = mv::paged_decode_cluster_kernel<T, D, NT, kMmaWarps, STAGES>;
    int rc = ensure_smem(kernel, Shape::kSmemBytes);
    if (rc != MV_OK) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(csize, p.kv_heads, p.batch);
    cfg.blockDim = dim3(kMmaWarps * 32);
    cfg.dynamicSmemBytes = Shape::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = csize;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t err = cudaLaunchKernelEx(&cfg, kernel, p, kmap, vmap);
    return err == cudaSuccess ? MV_OK : cuda_fail(err, "cluster decode kernel launch");
}

template <typename T>
int launch_cluster_dispatch(const mv::DecodeParams& p, const CUtensorMap& kmap, const CUtensorMap& vmap,
                            int csize, int nt, cudaStream_t stream) {
    switch (p.head_dim * 4 + nt) {
        case 64 * 4 + 1: return launch_cluster<T, 64, 1>(p, kmap, vmap, csize, stream);
        case 64 * 4 + 2: return launch_cluster<T, 64, 2>(p, kmap, vmap, csize, stream);
        case 128 * 4 + 1: return launch_cluster<T, 128, 1>(p, kmap, vmap, csize, stream);
        case 128 * 4 + 2: return launch_cluster<T, 128, 2>(p, kmap, vmap, csize, stream);
        case 256 * 4 + 1: return launch_cluster<T, 256, 1>(p, kmap, vmap, csize, stream);
        case 256 * 4 + 2: return launch_cluster<T, 256, 2>(p, kmap, vmap, csize, stream);
        default: return fail(MV_ERR_UNSUPPORTED, "no tensor-core kernel for head_dim %d", p.head_dim);
    }
}

template <typename T>
int launch_decode(const mv::DecodeParams& p, const Plan& plan, const CUtensorMap* kmap,
                  const CUtensorMap* vmap, cudaStream_t stream) {
    if (plan.path == MV_PATH_TMA_MMA_CLUSTER) {
        if constexpr (std::is_same<T, float>::value) {
            return fail(MV_ERR_UNSUPPORTED, "tensor-core kernel takes fp16/bf16 only");
        } else {
            return launch_cluster_dispatch<T>(p, *kmap, *vmap, plan.cluster, plan.nt, stream);
        }
    }
    if (plan.path == MV_PATH_TMA_MMA_PERSISTENT) {
        if constexpr (std::is_same<T, float>::value) {
            return fail(MV_ERR_UNSUPPORTED, "tensor-core kernel takes fp16/bf16 only");
        } else {
            return launch_persistent_dispatch<T>(p, *kmap, *vmap, plan.ctas, plan.nt, stream);
        }
    }
    if (plan.path == MV_PATH_TMA_MMA_STREAM) {
        if constexpr (std::is_same<T, float>::value) {
            return fail(MV_ERR_UNSUPPORTED, "tensor-core kernel takes fp16/bf16 only");
        } else {
            int rc = p.head_dim == 64 ? launch_stream<T, 64>(p, *kmap, *vmap, plan.ctas, stream)
                                      : launch_stream<T, 128>(p, *kmap, *vmap, plan.ctas, stream);
            if (rc != MV_OK) return rc;
            if (plan.max_splits > 1) {
                cudaError_t err = launch_split_merge<T>(p, stream);
                if (err != cudaSuccess) return cuda_fail(err, "merge kernel launch");
            }
            return MV_OK;
        }
    }
    const dim3 grid(plan.max_splits, p.kv_heads, p.batch);
    int rc;
    if (plan.path == MV_PATH_TMA_MMA) {
        if constexpr (std::is_same<T, float>::value) {
            return fail(MV_ERR_UNSUPPORTED, "tensor-core kernel takes fp16/bf16 only");
        } else {
            rc = launch_mma_dispatch<T>(p, *kmap, *vmap, grid, plan.nt, plan.wide, plan.cuda_core, stream);
        }
    } else {
        const size_t smem = mv::simt_smem_bytes(p.group, p.head_dim);
        auto kernel = mv::paged_decode_simt_kernel<T>;
        rc = ensure_smem(kernel, smem);
        if (rc == MV_OK) {
            cudaError_t err = launch_pdl(kernel, grid, dim3(mv::kSimtThreads), smem, stream, p);
            if (err != cudaSuccess) return cuda_fail(err, "decode kernel launch");
        }
    }
    if (rc != MV_OK) return rc;
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return cuda_fail(err, "decode kernel launch");
    if (plan.max_splits > 1 && !plan.fused_merge) {
        // Per output row: measured on B200, many short rows merge faster than
        // one CTA per (sequence, KV head) looping over its G rows.
        err = launch_split_merge<T>(p, stream);
        if (err != cudaSuccess) return cuda_fail(err, "merge kernel launch");
    }
    return MV_OK;
}

int check_index_type(int32_t type, const char* what) {
    if (type != MV_INDEX_I32 && type != MV_INDEX_I64)
        return fail(MV_ERR_INVALID_ARGUMENT, "%s type must be MV_INDEX_I32 or MV_INDEX_I64", what);
    return MV_OK;
}

size_t dtype_bytes(int32_t dtype) { return dtype == MV_DTYPE_F32 ? 4 : 2; }

// A contiguous cache can be read with TMA when its base is 16-byte aligned and
// the token, head and sequence strides in use are positive multiples of 16 bytes.
bool contiguous_tma_ok(const void* base, const int64_t* s, int heads, int batch) {
    if (reinterpret_cast<uintptr_t>(base) % 16) return false;
    if (s[2] <= 0 || (s[2] * 2) % 16) return false;
    if (heads > 1 && (s[1] <= 0 || (s[1] * 2) % 16)) return false;
    if (batch > 1 && (s[0] <= 0 || (s[0] * 2) % 16)) return false;
    return true;
}

// Strides of a dimension of extent 1 are never used: give the tensor map a valid one.
void contiguous_map_strides(const int64_t* s, int heads, int batch, int64_t tokens, int64_t* out) {
    out[0] = s[2];
    out[1] = heads > 1 ? s[1] : s[2] * ((tokens + 7) / 8 * 8);
    out[2] = batch > 1 ? s[0] : out[1] * heads;
}

// A chunk runs on the split grid (query tiles or rows), never the persistent,
// cluster or opted-in wide schedules, and merges in a separate pass.
uint32_t chunk_flags(uint32_t flags) {
    return flags & ~(MV_FLAG_PERSISTENT | MV_FLAG_CLUSTER | MV_FLAG_WIDE | MV_FLAG_FUSED_MERGE);
}

// Query tiles of chunk rows on tensor cores, then the split merge.
template <typename T>
int launch_chunk_tiles(const mv::DecodeParams& p, const Plan& plan, const CUtensorMap& kmap, const CUtensorMap& vmap,
                       int sequences, bool umma, cudaStream_t stream) {
    const int tile_rows = umma ? mv::kUmmaRows : mv::kChunkRows;
    const int q_tiles = (p.q_tokens * p.group + tile_rows - 1) / tile_rows;
    const dim3 grid(static_cast<unsigned>(q_tiles) * plan.max_splits, p.kv_heads, sequences);
    cudaError_t err;
    CUtensorMap khalf;
    if (umma) {
        const int dtype = std::is_same<T, __half>::value ? MV_DTYPE_F16 : MV_DTYPE_BF16;
        int rc = page_half_tensor_map(p.k_cache, p.num_blocks, p.kv_heads, p.head_dim, dtype, &khalf);
        if (rc != MV_OK) return rc;
    }
    if (umma && p.head_dim == 64) {
        auto kernel = mv::paged_chunk_umma_kernel<T, 64>;
        int rc = ensure_smem_carveout(kernel, mv::UmmaShape<64>::kSmemBytes);
        if (rc != MV_OK) return rc;
        err = launch_pdl(kernel, grid, dim3(mv::kUmmaThreads), mv::UmmaShape<64>::kSmemBytes, stream, p, khalf, vmap,
                         q_tiles);
    } else if (umma) {
        auto kernel = mv::paged_chunk_umma_kernel<T, 128>;
        int rc = ensure_smem_carveout(kernel, mv::UmmaShape<128>::kSmemBytes);
        if (rc != MV_OK) return rc;
        err = launch_pdl(kernel, grid, dim3(mv::kUmmaThreads), mv::UmmaShape<128>::kSmemBytes, stream, p, khalf,
                         vmap, q_tiles);
    } else if (p.head_dim == 64) {
        auto kernel = mv::paged_chunk_mma_kernel<T, 64>;
        int rc = ensure_smem_carveout(kernel, mv::ChunkShape<64>::kSmemBytes);
        if (rc != MV_OK) return rc;
        err = launch_pdl(kernel, grid, dim3(mv::kChunkThreads), mv::ChunkShape<64>::kSmemBytes, stream, p, kmap, vmap,
                         q_tiles);
    } else {
        auto kernel = mv::paged_chunk_mma_kernel<T, 128>;
        int rc = ensure_smem_carveout(kernel, mv::ChunkShape<128>::kSmemBytes);
        if (rc != MV_OK) return rc;
        err = launch_pdl(kernel, grid, dim3(mv::kChunkThreads), mv::ChunkShape<128>::kSmemBytes, stream, p, kmap,
                         vmap, q_tiles);
    }
    if (err != cudaSuccess) return cuda_fail(err, "chunk attention kernel launch");
    if (plan.max_splits > 1) {
        err = launch_split_merge<T>(p, stream);
        if (err != cudaSuccess) return cuda_fail(err, "merge kernel launch");
    }
    return MV_OK;
}

struct ContiguousCall {
    const void* k_cache;
    int64_t k_stride[3];  // sequence, head, token (elements)
    const void* v_cache;
    int64_t v_stride[3];
    int64_t cache_len;
};

int contiguous_plan(const ContiguousCall& c, int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                    int32_t head_dim, int64_t max_context_len, int32_t pages_per_split, uint32_t flags,
                    int32_t dtype, Plan* plan) {
    if (!c.k_cache || !c.v_cache) return fail(MV_ERR_INVALID_ARGUMENT, "k_cache and v_cache must not be NULL");
    if (c.cache_len <= 0) return fail(MV_ERR_INVALID_ARGUMENT, "cache_len must be positive");
    for (int i = 0; i < 3; ++i)
        if (c.k_stride[i] < 0 || c.v_stride[i] < 0) return fail(MV_ERR_INVALID_ARGUMENT, "strides must be nonnegative");
    if (max_context_len < 0) return fail(MV_ERR_INVALID_ARGUMENT, "max_context_len must be nonnegative");
    const int64_t bound = std::min(max_context_len, c.cache_len);
    const Geometry g{batch, num_q_heads, num_kv_heads, head_dim, 16, bound, dtype};
    const bool tma = contiguous_tma_ok(c.k_cache, c.k_stride, num_kv_heads, batch) &&
                     contiguous_tma_ok(c.v_cache, c.v_stride, num_kv_heads, batch);
    // The split grid and the CUDA-core kernel read contiguous caches; the
    // persistent and cluster schedules do not.
    return make_plan(g, pages_per_split, flags & ~(MV_FLAG_PERSISTENT | MV_FLAG_CLUSTER), tma, plan);
}

}  // namespace

extern "C" {

int mv_abi_version(void) { return MV_ABI_VERSION; }

const char* mv_last_error(void) { return g_error.c_str(); }

int mv_paged_decode_workspace_size(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads,
                                   int32_t head_dim, int32_t block_size, int64_t max_context_len,
                                   int32_t pages_per_split, uint32_t flags, int32_t dtype,
                                   size_t* bytes) {
    if (!bytes) return fail(MV_ERR_INVALID_ARGUMENT, "bytes must not be NULL");
    const Geometry g{batch, num_q_heads, num_kv_heads, head_dim, block_size, max_context_len, dtype};
    Plan plan;
    // Alignment never changes the split shape, so plan as if aligned.
    int rc = make_plan(g, pages_per_split, flags, true, &plan, StreamUse::kAllowed);
    if (rc != MV_OK) return rc;
    *bytes = plan.workspace;
    return MV_OK;
}

int mv_paged_chunk_workspace_size(int32_t batch, int32_t num_tokens, int32_t num_q_heads, int32_t num_kv_heads,
                                  int32_t head_dim, int32_t block_size, int64_t max_context_len,
                                  int32_t pages_per_split, uint32_t flags, int32_t dtype, size_t* bytes) {
    if (!bytes) return fail(MV_ERR_INVALID_ARGUMENT, "bytes must not be NULL");
    if (num_tokens <= 0 || batch <= 0) return fail(MV_ERR_INVALID_ARGUMENT, "batch and num_tokens must be positive");
    if (static_cast<int64_t>(batch) * num_tokens > 65535)
        return fail(MV_ERR_UNSUPPORTED, "batch x num_tokens is limited to 65535 query rows");
    const Geometry g{batch * num_tokens, num_q_heads, num_kv_heads, head_dim, block_size, max_context_len, dtype};
    Plan plan;
    bool tiles = false;
    int rc = make_chunk_plan(g, num_tokens, pages_per_split, chunk_flags(flags), true, &plan, &tiles);
    if (rc != MV_OK) return rc;
    *bytes = plan.workspace;
    return MV_OK;
}

int mv_paged_decode_plan(int32_t batch, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                         int32_t block_size, int64_t max_context_len, int32_t pages_per_split,
                         uint32_t flags, int32_t dtype, const void* k_cache, const void* v_cache,
                         int32_t* path, int32_t* chosen_pages_per_split, int32_t* max_splits) {
    const Geometry g{batch, num_q_heads, num_kv_heads, head_dim, block_size, max_context_len, dtype};
    Plan plan;
    int rc = make_plan(g, pages_per_split, flags, tma_aligned(k_cache, v_cache), &plan, StreamUse::kAllowed);
    if (rc != MV_OK) return rc;
    if (path) *path = plan.path;
    if (chosen_pages_per_split) *chosen_pages_per_split = plan.pages_per_split;
    if (max_splits) *max_splits = plan.max_splits;
    return MV_OK;
}

// This step's new K/V rows for mv_paged_decode_append ([batch, kv_heads], feature stride 1).
// A chunk of several new tokens per sequence (rows = batch x num_tokens).
struct ChunkRows {
    int32_t num_tokens;
    int64_t q_stride_token;
    int64_t out_stride_token;
};

struct NewRows {
    const void* key;
    int64_t key_stride_seq;
    int64_t key_stride_head;
    const void* value;
    int64_t value_stride_seq;
    int64_t value_stride_head;
    const void* rope_cos;  // nullptr: the rows and q are already rotated
    const void* rope_sin;
    int64_t rope_rows;
};

static int paged_decode_impl(const void* q, int64_t q_stride_seq, int64_t q_stride_head, const void* k_cache,
                    const void* v_cache, int64_t num_blocks, int32_t num_kv_heads, int32_t block_size,
                    int32_t head_dim, const void* block_table, int32_t block_table_type,
                    int64_t block_table_stride, int64_t blocks_per_seq, const void* context_lens,
                    int32_t context_lens_type, int64_t max_context_len, int32_t batch,
                    int32_t num_q_heads, float scale, void* out, int64_t out_stride_seq,
                    int64_t out_stride_head, void* workspace, size_t workspace_bytes,
                    int32_t pages_per_split, uint32_t flags, int32_t dtype, void* stream,
                             const NewRows* rows, const ChunkRows* chunk = nullptr) {
    if (!q || !k_cache || !v_cache || !block_table || !out)
        return fail(MV_ERR_INVALID_ARGUMENT, "q, k_cache, v_cache, block_table and out must not be NULL");
    if (num_blocks <= 0 || blocks_per_seq <= 0)
        return fail(MV_ERR_INVALID_ARGUMENT, "num_blocks and blocks_per_seq must be positive");
    if (num_blocks >= (int64_t(1) << 31)) return fail(MV_ERR_UNSUPPORTED, "num_blocks must be below 2^31");
    if (q_stride_seq < 0 || q_stride_head < 0 || out_stride_seq < 0 || out_stride_head < 0 ||
        block_table_stride < 0)
        return fail(MV_ERR_INVALID_ARGUMENT, "strides must be nonnegative");
    const int32_t tokens = chunk ? chunk->num_tokens : 1;
    const int32_t sequences = batch / tokens;  // `batch` counts query rows
    if (sequences > 1 && block_table_stride < blocks_per_seq)
        return fail(MV_ERR_INVALID_ARGUMENT, "block_table_stride is smaller than blocks_per_seq");
    int rc = check_index_type(block_table_type, "block_table");
    if (rc == MV_OK && context_lens) rc = check_index_type(context_lens_type, "context_lens");
    if (rc != MV_OK) return rc;
    if (!context_lens && max_context_len <= 0)
        return fail(MV_ERR_INVALID_ARGUMENT, "context length must be positive");
    if (!(scale == scale) || scale == INFINITY || scale == -INFINITY)
        return fail(MV_ERR_INVALID_ARGUMENT, "scale must be finite");

    const Geometry g{batch, num_q_heads, num_kv_heads, head_dim, block_size, max_context_len, dtype};
    Plan plan;
    bool tiles = false;
    rc = chunk ? make_chunk_plan(g, tokens, pages_per_split, flags, tma_aligned(k_cache, v_cache), &plan, &tiles)
               : make_plan(g, pages_per_split, flags, tma_aligned(k_cache, v_cache), &plan, StreamUse::kAllowed);
    if (rc != MV_OK) return rc;
    if (plan.workspace > 0 && (!workspace || workspace_bytes < plan.workspace))
        return fail(MV_ERR_WORKSPACE_TOO_SMALL, "workspace of %zu bytes needed, %zu given", plan.workspace,
                    workspace ? workspace_bytes : static_cast<size_t>(0));
    if (plan.workspace > 0 && reinterpret_cast<uintptr_t>(workspace) % 16)
        return fail(MV_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");

    mv::DecodeParams p{};
    p.q = q;
    p.q_stride_seq = q_stride_seq;
    p.q_stride_head = q_stride_head;
    p.k_cache = k_cache;
    p.v_cache = v_cache;
    p.num_blocks = num_blocks;
    p.kv_heads = num_kv_heads;
    p.block_size = block_size;
    p.head_dim = head_dim;
    p.group = num_q_heads / num_kv_heads;
    p.q_heads = num_q_heads;
    p.batch = batch;
    p.block_table = block_table;
    p.table_i64 = block_table_type == MV_INDEX_I64;
    p.table_stride = block_table_stride;
    p.blocks_per_seq = blocks_per_seq;
    p.context_lens = context_lens;
    p.lens_i64 = context_lens_type == MV_INDEX_I64;
    p.uniform_len = max_context_len;
    p.max_context_len = max_context_len;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.out_stride_seq = out_stride_seq;
    p.out_stride_head = out_stride_head;
    p.pages_per_split = plan.pages_per_split;
    p.max_splits = plan.max_splits;
    p.first_pages = plan.first_pages;
    p.later_pages = plan.later_pages;
    p.part_o = nullptr;
    p.part_lse = nullptr;
    p.prefix_out = nullptr;
    p.counters = nullptr;
    p.persistent_warps = plan.warps;
    p.fused_merge = plan.fused_merge ? 1 : 0;
    if (plan.workspace > 0) {
        uint8_t* base = static_cast<uint8_t*>(workspace);
        if (plan.counter_bytes > 0) p.counters = reinterpret_cast<unsigned*>(base);
        base += plan.counter_bytes;
        p.part_o = reinterpret_cast<float*>(base);
        p.part_lse = reinterpret_cast<float*>(base + plan.part_o_bytes);
        if (plan.path == MV_PATH_TMA_MMA_PERSISTENT)
            p.prefix_out = reinterpret_cast<int64_t*>(base + plan.part_o_bytes + plan.part_lse_bytes);
    }

    p.new_key = nullptr;
    p.new_value = nullptr;
    p.new_key_stride[0] = p.new_key_stride[1] = 0;
    p.new_value_stride[0] = p.new_value_stride[1] = 0;
    p.rope_cos = nullptr;
    p.rope_sin = nullptr;
    p.rope_rows = 0;
    p.contiguous = 0;
    for (int i = 0; i < 3; ++i) p.k_stride[i] = p.v_stride[i] = 0;
    p.q_tokens = tokens;
    p.q_stride_token = chunk ? chunk->q_stride_token : 0;
    p.out_stride_token = chunk ? chunk->out_stride_token : 0;
    if (rows) {
        // The split-grid tensor-core kernel (16-byte chunks) and the CUDA-core
        // kernel (elements) write the rows themselves; the persistent and
        // cluster schedules, and unaligned rows on the tensor-core path, run the
        // append kernel first, as two launches.
        const uintptr_t bits = reinterpret_cast<uintptr_t>(rows->key) | reinterpret_cast<uintptr_t>(rows->value) |
                               static_cast<uintptr_t>((rows->key_stride_seq | rows->key_stride_head |
                                                       rows->value_stride_seq | rows->value_stride_head) * 2);
        const bool fusable = ((plan.path == MV_PATH_TMA_MMA || plan.path == MV_PATH_TMA_MMA_STREAM) && bits % 16 == 0) ||
                             plan.path == MV_PATH_SIMT;
        if (rows->rope_cos) {
            const bool tables_ok = plan.path == MV_PATH_SIMT ||
                                   (reinterpret_cast<uintptr_t>(rows->rope_cos) |
                                    reinterpret_cast<uintptr_t>(rows->rope_sin)) % 16 == 0;
            if (!fusable || !tables_ok || head_dim % 2)
                return fail(MV_ERR_UNSUPPORTED,
                            "RoPE fusion needs the split grid or the CUDA-core kernel, an even head_dim and, on the "
                            "tensor-core path, 16-byte aligned K/V rows and tables; rotate with mv_apply_rope and "
                            "call without tables");
            p.rope_cos = rows->rope_cos;
            p.rope_sin = rows->rope_sin;
            p.rope_rows = rows->rope_rows;
        }
        if (fusable) {
            p.new_key = rows->key;
            p.new_value = rows->value;
            p.new_key_stride[0] = rows->key_stride_seq;
            p.new_key_stride[1] = rows->key_stride_head;
            p.new_value_stride[0] = rows->value_stride_seq;
            p.new_value_stride[1] = rows->value_stride_head;
        } else {
            rc = mv_write_paged_kv(rows->key, rows->key_stride_seq, rows->key_stride_head, 0, rows->value,
                                   rows->value_stride_seq, rows->value_stride_head, 0, const_cast<void*>(k_cache),
                                   const_cast<void*>(v_cache), num_blocks, num_kv_heads, block_size, head_dim,
                                   block_table, block_table_type, block_table_stride, blocks_per_seq,
                                   context_lens, context_lens_type, MV_POSITIONS_END,
                                   context_lens ? 0 : max_context_len - 1, batch, 1, dtype, stream);
            if (rc != MV_OK) return rc;
        }
    }

    CUtensorMap kmap, vmap;
    if (plan.path == MV_PATH_TMA_MMA || plan.path == MV_PATH_TMA_MMA_PERSISTENT ||
        plan.path == MV_PATH_TMA_MMA_CLUSTER || plan.path == MV_PATH_TMA_MMA_STREAM) {
        rc = page_tensor_map(k_cache, num_blocks, num_kv_heads, head_dim, dtype, &kmap);
        if (rc == MV_OK) rc = page_tensor_map(v_cache, num_blocks, num_kv_heads, head_dim, dtype, &vmap);
        if (rc != MV_OK) return rc;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // Chunks of tokens as query tiles on tensor cores where the chunk plan
    // allows them and the query's element pairs are 4-byte aligned.
    if (tiles && reinterpret_cast<uintptr_t>(q) % 4 == 0 &&
        ((q_stride_seq | q_stride_head | chunk->q_stride_token) & 1) == 0) {
        // tcgen05 tiles load 16-byte pieces of query rows.
        const bool umma = plan.chunk_umma && reinterpret_cast<uintptr_t>(q) % 16 == 0 &&
                          ((q_stride_seq | q_stride_head | chunk->q_stride_token) & 7) == 0;
        return dtype == MV_DTYPE_F16 ? launch_chunk_tiles<__half>(p, plan, kmap, vmap, sequences, umma, s)
                                     : launch_chunk_tiles<__nv_bfloat16>(p, plan, kmap, vmap, sequences, umma, s);
    }
    switch (dtype) {
        case MV_DTYPE_F32: return launch_decode<float>(p, plan, &kmap, &vmap, s);
        case MV_DTYPE_F16: return launch_decode<__half>(p, plan, &kmap, &vmap, s);
        default: return launch_decode<__nv_bfloat16>(p, plan, &kmap, &vmap, s);
    }
}

int mv_paged_decode(const void* q, int64_t q_stride_seq, int64_t q_stride_head, const void* k_cache,
                    const void* v_cache, int64_t num_blocks, int32_t num_kv_heads, int32_t block_size,
                    int32_t head_dim, const void* block_table, int32_t block_table_type,
                    int64_t block_table_stride, int64_t blocks_per_seq, const void* context_lens,
                    int32_t context_lens_type, int64_t max_context_len, int32_t batch,
                    int32_t num_q_heads, float scale, void* out, int64_t out_stride_seq,
                    int64_t out_stride_head, void* workspace, size_t workspace_bytes,
                    int32_t pages_per_split, uint32_t flags, int32_t dtype, void* stream) {
    return paged_decode_impl(q, q_stride_seq, q_stride_head, k_cache, v_cache, num_blocks, num_kv_heads,
                             block_size, head_dim, block_table, block_table_type, block_table_stride,
                             blocks_per_seq, context_lens, context_lens_type, max_context_len, batch,
                             num_q_heads, scale, out, out_stride_seq, out_stride_head, workspace,
                             workspace_bytes, pages_per_split, flags, dtype, stream, nullptr);
}

int mv_paged_decode_append(const void* q, int64_t q_stride_seq, int64_t q_stride_head, const void* key,
                           int64_t key_stride_seq, int64_t key_stride_head, const void* value,
                           int64_t value_stride_seq, int64_t value_stride_head, const void* rope_cos,
                           const void* rope_sin, int64_t rope_rows, void* k_cache, void* v_cache,
                           int64_t num_blocks, int32_t num_kv_heads, int32_t block_size, int32_t head_dim,
                           const void* block_table, int32_t block_table_type, int64_t block_table_stride,
                           int64_t blocks_per_seq, const void* context_lens, int32_t context_lens_type,
                           int64_t max_context_len, int32_t batch, int32_t num_q_heads, float scale, void* out,
                           int64_t out_stride_seq, int64_t out_stride_head, void* workspace,
                           size_t workspace_bytes, int32_t pages_per_split, uint32_t flags, int32_t dtype,
                           void* stream) {
    if (!key || !value) return fail(MV_ERR_INVALID_ARGUMENT, "key and value must not be NULL");
    if (key_stride_seq < 0 || key_stride_head < 0 || value_stride_seq < 0 || value_stride_head < 0)
        return fail(MV_ERR_INVALID_ARGUMENT, "strides must be nonnegative");
    if ((rope_cos == nullptr) != (rope_sin == nullptr))
        return fail(MV_ERR_INVALID_ARGUMENT, "pass both RoPE tables or neither");
    if (rope_cos && rope_rows <= 0) return fail(MV_ERR_INVALID_ARGUMENT, "rope_rows must be positive");
    const NewRows rows{key, key_stride_seq, key_stride_head, value, value_stride_seq, value_stride_head,
                       rope_cos, rope_sin, rope_rows};
    return paged_decode_impl(q, q_stride_seq, q_stride_head, k_cache, v_cache, num_blocks, num_kv_heads,
                             block_size, head_dim, block_table, block_table_type, block_table_stride,
                             blocks_per_seq, context_lens, context_lens_type, max_context_len, batch,
                             num_q_heads, scale, out, out_stride_seq, out_stride_head, workspace,
                             workspace_bytes, pages_per_split, flags, dtype, stream, &rows);
}

int mv_paged_decode_step_args(const MvDecodeStepArgs* a, void* stream) {
    if (!a) return fail(MV_ERR_INVALID_ARGUMENT, "args must not be NULL");
    const int64_t narrow[] = {a->num_kv_heads, a->block_size, a->head_dim, a->block_table_type,
                              a->context_lens_type, a->batch, a->num_q_heads, a->pages_per_split, a->dtype};
    for (const int64_t v : narrow)
        if (v < INT32_MIN || v > INT32_MAX) return fail(MV_ERR_INVALID_ARGUMENT, "an int32 field is out of range");
    if (a->flags > UINT32_MAX) return fail(MV_ERR_INVALID_ARGUMENT, "flags out of range");
    const uint32_t flags = static_cast<uint32_t>(a->flags);
    if (!a->key && !a->value)
        return mv_paged_decode(a->q, a->q_stride_seq, a->q_stride_head, a->k_cache, a->v_cache, a->num_blocks,
                               static_cast<int32_t>(a->num_kv_heads), static_cast<int32_t>(a->block_size),
                               static_cast<int32_t>(a->head_dim), a->block_table,
                               static_cast<int32_t>(a->block_table_type), a->block_table_stride, a->blocks_per_seq,
                               a->context_lens, static_cast<int32_t>(a->context_lens_type), a->max_context_len,
                               static_cast<int32_t>(a->batch), static_cast<int32_t>(a->num_q_heads),
                               static_cast<float>(a->scale), a->out, a->out_stride_seq, a->out_stride_head,
                               a->workspace, a->workspace_bytes, static_cast<int32_t>(a->pages_per_split), flags,
                               static_cast<int32_t>(a->dtype), stream);
    return mv_paged_decode_append(a->q, a->q_stride_seq, a->q_stride_head, a->key, a->key_stride_seq,
                                  a->key_stride_head, a->value, a->value_stride_seq, a->value_stride_head,
                                  a->rope_cos, a->rope_sin, a->rope_rows, a->k_cache, a->v_cache, a->num_blocks,
                                  static_cast<int32_t>(a->num_kv_heads), static_cast<int32_t>(a->block_size),
                                  static_cast<int32_t>(a->head_dim), a->block_table,
                                  static_cast<int32_t>(a->block_table_type), a->block_table_stride,
                                  a->blocks_per_seq, a->context_lens, static_cast<int32_t>(a->context_lens_type),
                                  a->max_context_len, static_cast<int32_t>(a->batch),
                                  static_cast<int32_t>(a->num_q_heads), static_cast<float>(a->scale), a->out,
                                  a->out_stride_seq, a->out_stride_head, a->workspace, a->workspace_bytes,
                                  static_cast<int32_t>(a->pages_per_split), flags, static_cast<int32_t>(a->dtype),
                                  stream);
}

int mv_paged_chunk_attention(const void* q, int64_t q_stride_seq, int64_t q_stride_token, int64_t q_stride_head,
                             const void* k_cache, const void* v_cache, int64_t num_blocks, int32_t num_kv_heads,
                             int32_t block_size, int32_t head_dim, const void* block_table,
                             int32_t block_table_type, int64_t block_table_stride, int64_t blocks_per_seq,
                             const void* context_lens, int32_t context_lens_type, int64_t max_context_len,
                             int32_t batch, int32_t num_tokens, int32_t num_q_heads, float scale, void* out,
                             int64_t out_stride_seq, int64_t out_stride_token, int64_t out_stride_head,
                             void* workspace, size_t workspace_bytes, int32_t pages_per_split, uint32_t flags,
                             int32_t dtype, void* stream) {
    if (num_tokens <= 0 || batch <= 0) return fail(MV_ERR_INVALID_ARGUMENT, "batch and num_tokens must be positive");
    if (static_cast<int64_t>(batch) * num_tokens > 65535)
        return fail(MV_ERR_UNSUPPORTED, "batch x num_tokens is limited to 65535 query rows");
    if (q_stride_token < 0 || out_stride_token < 0) return fail(MV_ERR_INVALID_ARGUMENT, "strides must be nonnegative");
    const ChunkRows chunk{num_tokens, q_stride_token, out_stride_token};
    return paged_decode_impl(q, q_stride_seq, q_stride_head, k_cache, v_cache, num_blocks, num_kv_heads, block_size,
                             head_dim, block_table, block_table_type, block_table_stride, blocks_per_seq,
                             context_lens, context_lens_type, max_context_len, batch * num_tokens, num_q_heads,
                             scale, out, out_stride_seq, out_stride_head, workspace, workspace_bytes,
                             pages_per_split, chunk_flags(flags), dtype, stream, nullptr, &chunk);
}

int mv_contiguous_decode_plan(const void* k_cache, int64_t k_stride_seq, int64_t k_stride_head,
                              int64_t k_stride_token, const void* v_cache, int64_t v_stride_seq,
                              int64_t v_stride_head, int64_t v_stride_token, int64_t cache_len,
                              int32_t num_kv_heads, int32_t head_dim, int64_t max_context_len, int32_t batch,
                              int32_t num_q_heads, int32_t pages_per_split, uint32_t flags, int32_t dtype,
                              int32_t* path, int32_t* chosen_pages_per_split, int32_t* max_splits,
                              size_t* workspace_bytes) {
    if (!path || !chosen_pages_per_split || !max_splits || !workspace_bytes)
        return fail(MV_ERR_INVALID_ARGUMENT, "outputs must not be NULL");
    const ContiguousCall c{k_cache, {k_stride_seq, k_stride_head, k_stride_token},
                           v_cache, {v_stride_seq, v_stride_head, v_stride_token}, cache_len};
    Plan plan;
    int rc = contiguous_plan(c, batch, num_q_heads, num_kv_heads, head_dim, max_context_len, pages_per_split,
                             flags, dtype, &plan);
    if (rc != MV_OK) return rc;
    *path = plan.path;
    *chosen_pages_per_split = plan.pages_per_split;
    *max_splits = plan.max_splits;
    *workspace_bytes = plan.workspace;
    return MV_OK;
}

int mv_contiguous_decode(const void* q, int64_t q_stride_seq, int64_t q_stride_head, const void* k_cache,
                         int64_t k_stride_seq, int64_t k_stride_head, int64_t k_stride_token, const void* v_cache,
                         int64_t v_stride_seq, int64_t v_stride_head, int64_t v_stride_token, int64_t cache_len,
                         int32_t num_kv_heads, int32_t head_dim, const void* context_lens,
                         int32_t context_lens_type, int64_t max_context_len, int32_t batch, int32_t num_q_heads,
                         float scale, void* out, int64_t out_stride_seq, int64_t out_stride_head,
                         void* workspace, size_t workspace_bytes, int32_t pages_per_split, uint32_t flags,
                         int32_t dtype, void* stream) {
    if (!q || !out) return fail(MV_ERR_INVALID_ARGUMENT, "q and out must not be NULL");
    if (q_stride_seq < 0 || q_stride_head < 0 || out_stride_seq < 0 || out_stride_head < 0)
        return fail(MV_ERR_INVALID_ARGUMENT, "strides must be nonnegative");
    int rc = context_lens ? check_index_type(context_lens_type, "context_lens") : MV_OK;
    if (rc != MV_OK) return rc;
    if (!context_lens && max_context_len <= 0)
        return fail(MV_ERR_INVALID_ARGUMENT, "context length must be positive");
    if (!(scale == scale) || scale == INFINITY || scale == -INFINITY)
        return fail(MV_ERR_INVALID_ARGUMENT, "scale must be finite");
    const ContiguousCall c{k_cache, {k_stride_seq, k_stride_head, k_stride_token},
                           v_cache, {v_stride_seq, v_stride_head, v_stride_token}, cache_len};
    Plan plan;
    rc = contiguous_plan(c, batch, num_q_heads, num_kv_heads, head_dim, max_context_len, pages_per_split, flags,
                         dtype, &plan);
    if (rc != MV_OK) return rc;
    if (plan.workspace > 0 && (!workspace || workspace_bytes < plan.workspace))
        return fail(MV_ERR_WORKSPACE_TOO_SMALL, "workspace of %zu bytes needed, %zu given", plan.workspace,
                    workspace ? workspace_bytes : static_cast<size_t>(0));
    if (plan.workspace > 0 && reinterpret_cast<uintptr_t>(workspace) % 16)
        return fail(MV_ERR_INVALID_ARGUMENT, "workspace must be 16-byte aligned");

    const int64_t bound = std::min(max_context_len, cache_len);
    const int64_t runs = (cache_len + 15) / 16;  // 16-token runs stand in for pages
    mv::DecodeParams p{};
    std::memset(&p, 0, sizeof(p));
    p.q = q;
    p.q_stride_seq = q_stride_seq;
    p.q_stride_head = q_stride_head;
    p.k_cache = k_cache;
    p.v_cache = v_cache;
    p.num_blocks = runs;
    p.kv_heads = num_kv_heads;
    p.block_size = 16;
    p.head_dim = head_dim;
    p.group = num_q_heads / num_kv_heads;
    p.q_heads = num_q_heads;
    p.batch = batch;
    p.block_table = nullptr;
    p.blocks_per_seq = runs;
    p.context_lens = context_lens;
    p.lens_i64 = context_lens_type == MV_INDEX_I64;
    p.uniform_len = bound;
    p.max_context_len = bound;
    p.scale_log2 = scale * 1.4426950408889634f;
    p.out = out;
    p.out_stride_seq = out_stride_seq;
    p.out_stride_head = out_stride_head;
    p.pages_per_split = plan.pages_per_split;
    p.max_splits = plan.max_splits;
    p.first_pages = plan.first_pages;
    p.later_pages = plan.later_pages;
    p.fused_merge = plan.fused_merge ? 1 : 0;
    p.contiguous = 1;
    for (int i = 0; i < 3; ++i) {
        p.k_stride[i] = c.k_stride[i];
        p.v_stride[i] = c.v_stride[i];
    }
    if (plan.workspace > 0) {
        uint8_t* base = static_cast<uint8_t*>(workspace);
        if (plan.fused_merge || plan.path == MV_PATH_TMA_MMA_STREAM) p.counters = reinterpret_cast<unsigned*>(base);
        base += plan.counter_bytes;
        p.part_o = reinterpret_cast<float*>(base);
        p.part_lse = reinterpret_cast<float*>(base + plan.part_o_bytes);
    }
    CUtensorMap kmap, vmap;
    if (plan.path == MV_PATH_TMA_MMA) {
        int64_t ks[3], vs[3];
        contiguous_map_strides(c.k_stride, num_kv_heads, batch, cache_len, ks);
        contiguous_map_strides(c.v_stride, num_kv_heads, batch, cache_len, vs);
        rc = contiguous_tensor_map(k_cache, cache_len, num_kv_heads, batch, head_dim, ks, dtype, &kmap);
        if (rc == MV_OK) rc = contiguous_tensor_map(v_cache, cache_len, num_kv_heads, batch, head_dim, vs, dtype, &vmap);
        if (rc != MV_OK) return rc;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (dtype) {
        case MV_DTYPE_F32: return launch_decode<float>(p, plan, &kmap, &vmap, s);
        case MV_DTYPE_F16: return launch_decode<__half>(p, plan, &kmap, &vmap, s);
        default: return launch_decode<__nv_bfloat16>(p, plan, &kmap, &vmap, s);
    }
}

int mv_write_paged_kv(const void* key, int64_t key_stride_seq, int64_t key_stride_head,
                      int64_t key_stride_token, const void* value, int64_t value_stride_seq,
                      int64_t value_stride_head, int64_t value_stride_token, void* k_cache,
                      void* v_cache, int64_t num_blocks, int32_t num_kv_heads, int32_t block_size,
                      int32_t head_dim, const void* block_table, int32_t block_table_type,
                      int64_t block_table_stride, int64_t blocks_per_seq, const void* positions,
                      int32_t positions_type, int32_t positions_kind, int64_t start, int32_t batch,
                      int32_t num_tokens, int32_t dtype, void* stream) {
    if (!key || !value || !k_cache || !v_cache || !block_table)
        return fail(MV_ERR_INVALID_ARGUMENT, "key, value, caches and block_table must not be NULL");
    if (num_blocks <= 0 || num_kv_heads <= 0 || block_size <= 0 || head_dim <= 0 || blocks_per_seq <= 0 ||
        batch <= 0 || num_tokens <= 0)
        return fail(MV_ERR_INVALID_ARGUMENT, "sizes must be positive");
    if (dtype != MV_DTYPE_F32 && dtype != MV_DTYPE_F16 && dtype != MV_DTYPE_BF16)
        return fail(MV_ERR_INVALID_ARGUMENT, "dtype must be MV_DTYPE_F32, MV_DTYPE_F16 or MV_DTYPE_BF16");
    const int64_t strides[6] = {key_stride_seq, key_stride_head, key_stride_token,
                                value_stride_seq, value_stride_head, value_stride_token};
    for (int64_t s : strides)
        if (s < 0) return fail(MV_ERR_INVALID_ARGUMENT, "strides must be nonnegative");
    if (block_table_stride < 0) return fail(MV_ERR_INVALID_ARGUMENT, "block_table_stride must be nonnegative");
    if (batch > 1 && block_table_stride < blocks_per_seq)
        return fail(MV_ERR_INVALID_ARGUMENT, "block_table_stride is smaller than blocks_per_seq");
    int rc = check_index_type(block_table_type, "block_table");
    if (rc == MV_OK && positions) rc = check_index_type(positions_type, "positions");
    if (rc != MV_OK) return rc;
    if (positions && positions_kind != MV_POSITIONS_START && positions_kind != MV_POSITIONS_END)
        return fail(MV_ERR_INVALID_ARGUMENT, "positions_kind must be MV_POSITIONS_START or MV_POSITIONS_END");
    DeviceInfo dev;
    rc = device_info(&dev);
    if (rc != MV_OK) return rc;

    mv::AppendParams a;
    a.key = key;
    a.value = value;
    a.key_stride[0] = key_stride_seq;
    a.key_stride[1] = key_stride_head;
    a.key_stride[2] = key_stride_token;
    a.value_stride[0] = value_stride_seq;
    a.value_stride[1] = value_stride_head;
    a.value_stride[2] = value_stride_token;
    a.k_cache = k_cache;
    a.v_cache = v_cache;
    a.num_blocks = num_blocks;
    a.kv_heads = num_kv_heads;
    a.block_size = block_size;
    a.elem_bytes = static_cast<int>(dtype_bytes(dtype));
    a.row_bytes = head_dim * a.elem_bytes;
    a.block_table = block_table;
    a.table_i64 = block_table_type == MV_INDEX_I64;
    a.table_stride = block_table_stride;
    a.blocks_per_seq = blocks_per_seq;
    a.positions = positions;
    a.positions_i64 = positions_type == MV_INDEX_I64;
    a.positions_end = positions_kind == MV_POSITIONS_END;
    a.start = start;
    a.batch = batch;
    a.num_tokens = num_tokens;

    // Widest vector every address and stride allows.
    uintptr_t bits = reinterpret_cast<uintptr_t>(key) | reinterpret_cast<uintptr_t>(value) |
                     reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache) |
                     static_cast<uintptr_t>(a.row_bytes);
    for (int64_t s : strides) bits |= static_cast<uintptr_t>(s * a.elem_bytes);
    int vec = 16;
    while (vec > 2 && (bits % vec)) vec >>= 1;
    const int64_t total = static_cast<int64_t>(batch) * num_tokens * num_kv_heads * 2 * (a.row_bytes / vec);
    const int64_t want = (total + mv::kAppendThreads - 1) / mv::kAppendThreads;
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(dev.sms) * 16)));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaError_t err;
    const dim3 grid(blocks), block(mv::kAppendThreads);
    switch (vec) {
        case 16: err = launch_pdl(mv::write_paged_kv_kernel<16>, grid, block, 0, s, a, total); break;
        case 8: err = launch_pdl(mv::write_paged_kv_kernel<8>, grid, block, 0, s, a, total); break;
        case 4: err = launch_pdl(mv::write_paged_kv_kernel<4>, grid, block, 0, s, a, total); break;
        default: err = launch_pdl(mv::write_paged_kv_kernel<2>, grid, block, 0, s, a, total); break;
    }
    return err == cudaSuccess ? MV_OK : cuda_fail(err, "append kernel launch");
}

int mv_apply_rope(const void* x, int64_t x_stride_seq, int64_t x_stride_head, int64_t x_stride_token, void* out,
                  int64_t out_stride_seq, int64_t out_stride_head, int64_t out_stride_token, int32_t batch,
                  int32_t heads, int32_t num_tokens, int32_t head_dim, const void* cos, const void* sin,
                  int64_t table_rows, const void* positions, int32_t positions_type, int32_t positions_kind,
                  int64_t start, int32_t dtype, void* stream) {
    if (!x || !out || !cos || !sin) return fail(MV_ERR_INVALID_ARGUMENT, "x, out and the tables must not be NULL");
    if (batch <= 0 || heads <= 0 || num_tokens <= 0 || head_dim <= 0 || table_rows <= 0)
        return fail(MV_ERR_INVALID_ARGUMENT, "sizes must be positive");
    if (head_dim % 2) return fail(MV_ERR_INVALID_ARGUMENT, "head_dim must be even");
    if (dtype != MV_DTYPE_F32 && dtype != MV_DTYPE_F16 && dtype != MV_DTYPE_BF16)
        return fail(MV_ERR_INVALID_ARGUMENT, "dtype must be MV_DTYPE_F32, MV_DTYPE_F16 or MV_DTYPE_BF16");
    const int64_t strides[6] = {x_stride_seq, x_stride_head, x_stride_token,
                                out_stride_seq, out_stride_head, out_stride_token};
    for (int64_t s : strides)
        if (s < 0) return fail(MV_ERR_INVALID_ARGUMENT, "strides must be nonnegative");
    int rc = positions ? check_index_type(positions_type, "positions") : MV_OK;
    if (rc != MV_OK) return rc;
    if (positions && positions_kind != MV_POSITIONS_START && positions_kind != MV_POSITIONS_END)
        return fail(MV_ERR_INVALID_ARGUMENT, "positions_kind must be MV_POSITIONS_START or MV_POSITIONS_END");
    DeviceInfo dev;
    rc = device_info(&dev);
    if (rc != MV_OK) return rc;
    mv::RopeParams r;
    r.x = x;
    r.x_stride[0] = x_stride_seq;
    r.x_stride[1] = x_stride_head;
    r.x_stride[2] = x_stride_token;
    r.out = out;
    r.out_stride[0] = out_stride_seq;
    r.out_stride[1] = out_stride_head;
    r.out_stride[2] = out_stride_token;
    r.batch = batch;
    r.heads = heads;
    r.tokens = num_tokens;
    r.head_dim = head_dim;
    r.cos = cos;
    r.sin = sin;
    r.table_rows = table_rows;
    r.positions = positions;
    r.positions_i64 = positions_type == MV_INDEX_I64;
    r.positions_end = positions_kind == MV_POSITIONS_END;
    r.start = start;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 block(mv::kRopeThreads);
    cudaError_t err;
    // Two-byte rows of a multiple of 16 elements, everything 16-byte aligned: 16-byte chunks.
    uintptr_t bits = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(out) |
                     reinterpret_cast<uintptr_t>(cos) | reinterpret_cast<uintptr_t>(sin);
    for (int64_t st : strides) bits |= static_cast<uintptr_t>(st * 2);
    const int64_t row_chunks = static_cast<int64_t>(num_tokens) * (head_dim / 16);
    if (dtype != MV_DTYPE_F32 && head_dim % 16 == 0 && bits % 16 == 0 && heads <= 65535 && batch <= 65535 &&
        row_chunks < (int64_t(1) << 30)) {
        const dim3 grid(static_cast<unsigned>((row_chunks + mv::kRopeThreads - 1) / mv::kRopeThreads), heads, batch);
        err = dtype == MV_DTYPE_F16 ? launch_pdl(mv::rope_rows_vec_kernel<__half>, grid, block, 0, s, r)
                                    : launch_pdl(mv::rope_rows_vec_kernel<__nv_bfloat16>, grid, block, 0, s, r);
        return err == cudaSuccess ? MV_OK : cuda_fail(err, "RoPE kernel launch");
    }
    const int64_t total = static_cast<int64_t>(batch) * heads * num_tokens * (head_dim / 2);
    const int64_t want = (total + mv::kRopeThreads - 1) / mv::kRopeThreads;
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(dev.sms) * 16)));
    const dim3 grid(blocks);
    switch (dtype) {
        case MV_DTYPE_F32: err = launch_pdl(mv::rope_rows_kernel<float>, grid, block, 0, s, r, total); break;
        case MV_DTYPE_F16: err = launch_pdl(mv::rope_rows_kernel<__half>, grid, block, 0, s, r, total); break;
        default: err = launch_pdl(mv::rope_rows_kernel<__nv_bfloat16>, grid, block, 0, s, r, total); break;
    }
    return err == cudaSuccess ? MV_OK : cuda_fail(err, "RoPE kernel launch");
}

int mv_rms_norm(const void* x, int64_t x_stride_row, const void* weight, void* out, int64_t out_stride_row,
                int64_t rows, int32_t hidden, float eps, int32_t dtype, void* stream) {
    if (!x || !weight || !out) return fail(MV_ERR_INVALID_ARGUMENT, "x, weight and out must not be NULL");
    if (rows <= 0 || hidden <= 0) return fail(MV_ERR_INVALID_ARGUMENT, "sizes must be positive");
    if (rows >= (int64_t(1) << 31)) return fail(MV_ERR_UNSUPPORTED, "rows must be below 2^31");
    if (x_stride_row < hidden || out_stride_row < hidden)
        return fail(MV_ERR_INVALID_ARGUMENT, "row strides must cover the row");
    if (!(eps >= 0.0f) || eps == INFINITY) return fail(MV_ERR_INVALID_ARGUMENT, "eps must be finite and nonnegative");
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>(rows)), block(mv::kRowThreads);
    cudaError_t err;
    const size_t elem = dtype == MV_DTYPE_F32 ? 4 : 2;
    const int per_chunk = static_cast<int>(16 / elem);
    const uintptr_t bits = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(weight) |
                           reinterpret_cast<uintptr_t>(out) | static_cast<uintptr_t>(x_stride_row * elem) |
                           static_cast<uintptr_t>(out_stride_row * elem);
    DeviceInfo dev;
    int rc = device_info(&dev);
    if (rc != MV_OK) return rc;
    if (hidden % per_chunk == 0 && bits % 16 == 0 && hidden / per_chunk <= 32 * mv::kWarpNormChunks &&
        rows >= static_cast<int64_t>(dev.sms) * 8) {
        // Many rows that each fit a warp: one warp per row, eight rows per CTA
        // (measured on B200: 14.7 vs 29 us for 16384 x 1536). Few rows keep one
        // CTA per row, which spreads a small batch over more SMs (3.5 vs 6.1 us
        // for 32 x 1536).
        const dim3 wgrid(static_cast<unsigned>((rows + mv::kRowThreads / 32 - 1) / (mv::kRowThreads / 32)));
        switch (dtype) {
            case MV_DTYPE_F32:
                err = launch_pdl(mv::rms_norm_warp_kernel<float>, wgrid, block, 0, s, static_cast<const float*>(x),
                                 x_stride_row, static_cast<const float*>(weight), static_cast<float*>(out),
                                 out_stride_row, hidden, eps, rows);
                break;
            case MV_DTYPE_F16:
                err = launch_pdl(mv::rms_norm_warp_kernel<__half>, wgrid, block, 0, s, static_cast<const __half*>(x),
                                 x_stride_row, static_cast<const __half*>(weight), static_cast<__half*>(out),
                                 out_stride_row, hidden, eps, rows);
                break;
            case MV_DTYPE_BF16:
                err = launch_pdl(mv::rms_norm_warp_kernel<__nv_bfloat16>, wgrid, block, 0, s,
                                 static_cast<const __nv_bfloat16*>(x), x_stride_row,
                                 static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out),
                                 out_stride_row, hidden, eps, rows);
                break;
            default: return fail(MV_ERR_INVALID_ARGUMENT, "dtype must be MV_DTYPE_F32, MV_DTYPE_F16 or MV_DTYPE_BF16");
        }
        return err == cudaSuccess ? MV_OK : cuda_fail(err, "RMSNorm kernel launch");
    }
    if (hidden % per_chunk == 0 && bits % 16 == 0 && hidden / per_chunk <= mv::kRowThreads * mv::kNormMaxChunks) {
        switch (dtype) {
            case MV_DTYPE_F32:
                err = launch_pdl(mv::rms_norm_vec_kernel<float>, grid, block, 0, s, static_cast<const float*>(x),
                                 x_stride_row, static_cast<const float*>(weight), static_cast<float*>(out),
                                 out_stride_row, hidden, eps);
                break;
            case MV_DTYPE_F16:
                err = launch_pdl(mv::rms_norm_vec_kernel<__half>, grid, block, 0, s, static_cast<const __half*>(x),
                                 x_stride_row, static_cast<const __half*>(weight), static_cast<__half*>(out),
                                 out_stride_row, hidden, eps);
                break;
            case MV_DTYPE_BF16:
                err = launch_pdl(mv::rms_norm_vec_kernel<__nv_bfloat16>, grid, block, 0, s,
                                 static_cast<const __nv_bfloat16*>(x), x_stride_row,
                                 static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out),
                                 out_stride_row, hidden, eps);
                break;
            default: return fail(MV_ERR_INVALID_ARGUMENT, "dtype must be MV_DTYPE_F32, MV_DTYPE_F16 or MV_DTYPE_BF16");
        }
        return err == cudaSuccess ? MV_OK : cuda_fail(err, "RMSNorm kernel launch");
    }
    switch (dtype) {
        case MV_DTYPE_F32:
            err = launch_pdl(mv::rms_norm_kernel<float>, grid, block, 0, s, static_cast<const float*>(x), x_stride_row,
                             static_cast<const float*>(weight), static_cast<float*>(out), out_stride_row, hidden, eps);
            break;
        case MV_DTYPE_F16:
            err = launch_pdl(mv::rms_norm_kernel<__half>, grid, block, 0, s, static_cast<const __half*>(x), x_stride_row,
                             static_cast<const __half*>(weight), static_cast<__half*>(out), out_stride_row, hidden, eps);
            break;
        case MV_DTYPE_BF16:
            err = launch_pdl(mv::rms_norm_kernel<__nv_bfloat16>, grid, block, 0, s,
                             static_cast<const __nv_bfloat16*>(x), x_stride_row,
                             static_cast<const __nv_bfloat16*>(weight), static_cast<__nv_bfloat16*>(out),
                             out_stride_row, hidden, eps);
            break;
        default: return fail(MV_ERR_INVALID_ARGUMENT, "dtype must be MV_DTYPE_F32, MV_DTYPE_F16 or MV_DTYPE_BF16");
    }
    return err == cudaSuccess ? MV_OK : cuda_fail(err, "RMSNorm kernel launch");
}

int mv_silu_mul(const void* gate_up, int64_t stride_row, void* out, int64_t out_stride_row, int64_t rows,
                int32_t width, int32_t dtype, void* stream) {
    if (!gate_up || !out) return fail(MV_ERR_INVALID_ARGUMENT, "gate_up and out must not be NULL");
    if (rows <= 0 || width <= 0) return fail(MV_ERR_INVALID_ARGUMENT, "sizes must be positive");
    if (stride_row < 2 * static_cast<int64_t>(width) || out_stride_row < width)
        return fail(MV_ERR_INVALID_ARGUMENT, "row strides must cover the row");
    DeviceInfo dev;
    int rc = device_info(&dev);
    if (rc != MV_OK) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 block(mv::kRowThreads);
    cudaError_t err;
    const size_t elem = dtype == MV_DTYPE_F32 ? 4 : 2;
    const int per_chunk = static_cast<int>(16 / elem);
    const uintptr_t bits = reinterpret_cast<uintptr_t>(gate_up) | reinterpret_cast<uintptr_t>(out) |
                           static_cast<uintptr_t>(stride_row * elem) | static_cast<uintptr_t>(out_stride_row * elem);
    if (width % per_chunk == 0 && bits % 16 == 0) {
        const int chunks = width / per_chunk;
        const dim3 grid((chunks + mv::kRowThreads - 1) / mv::kRowThreads,
                        static_cast<unsigned>(std::min<int64_t>(rows, 65535)));
        switch (dtype) {
            case MV_DTYPE_F32:
                err = launch_pdl(mv::silu_mul_vec_kernel<float>, grid, block, 0, s, static_cast<const float*>(gate_up),
                                 stride_row, static_cast<float*>(out), out_stride_row, static_cast<int>(width), rows);
                break;
            case MV_DTYPE_F16:
                err = launch_pdl(mv::silu_mul_vec_kernel<__half>, grid, block, 0, s,
                                 static_cast<const __half*>(gate_up), stride_row, static_cast<__half*>(out),
                                 out_stride_row, static_cast<int>(width), rows);
                break;
            case MV_DTYPE_BF16:
                err = launch_pdl(mv::silu_mul_vec_kernel<__nv_bfloat16>, grid, block, 0, s,
                                 static_cast<const __nv_bfloat16*>(gate_up), stride_row,
                                 static_cast<__nv_bfloat16*>(out), out_stride_row, static_cast<int>(width), rows);
                break;
            default: return fail(MV_ERR_INVALID_ARGUMENT, "dtype must be MV_DTYPE_F32, MV_DTYPE_F16 or MV_DTYPE_BF16");
        }
        return err == cudaSuccess ? MV_OK : cuda_fail(err, "SiLU-mul kernel launch");
    }
    const int64_t total = rows * width;
    const int64_t want = (total + mv::kRowThreads - 1) / mv::kRowThreads;
    const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(want, static_cast<int64_t>(dev.sms) * 16)));
    const dim3 grid(blocks);
    switch (dtype) {
        case MV_DTYPE_F32:
            err = launch_pdl(mv::silu_mul_kernel<float>, grid, block, 0, s, static_cast<const float*>(gate_up),
                             stride_row, static_cast<float*>(out), out_stride_row, static_cast<int>(width), total);
            break;
        case MV_DTYPE_F16:
            err = launch_pdl(mv::silu_mul_kernel<__half>, grid, block, 0, s, static_cast<const __half*>(gate_up),
                             stride_row, static_cast<__half*>(out), out_stride_row, static_cast<int>(width), total);
            break;
        case MV_DTYPE_BF16:
            err = launch_pdl(mv::silu_mul_kernel<__nv_bfloat16>, grid, block, 0, s,
                             static_cast<const __nv_bfloat16*>(gate_up), stride_row,
                             static_cast<__nv_bfloat16*>(out), out_stride_row, static_cast<int>(width), total);
            break;
        default: return fail(MV_ERR_INVALID_ARGUMENT, "dtype must be MV_DTYPE_F32, MV_DTYPE_F16 or MV_DTYPE_BF16");
    }
    return err == cudaSuccess ? MV_OK : cuda_fail(err, "SiLU-mul kernel launch");
}

int mv_device_status(int32_t device, uint32_t* status) {
    if (!status) return fail(MV_ERR_INVALID_ARGUMENT, "status must not be NULL");
    int prev = 0;
    cudaError_t err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != device) err = cudaSetDevice(device);
    unsigned int value = 0;
    if (err == cudaSuccess) err = cudaMemcpyFromSymbol(&value, mv::g_device_status, sizeof(value));
    if (prev != device) cudaSetDevice(prev);
    if (err != cudaSuccess) return cuda_fail(err, "reading device status");
    *status = value;
    return MV_OK;
}

int mv_clear_device_status(int32_t device) {
    int prev = 0;
    cudaError_t err = cudaGetDevice(&prev);
    if (err == cudaSuccess && prev != device) err = cudaSetDevice(device);
    const unsigned int zero = 0;
    if (err == cudaSuccess) err = cudaMemcpyToSymbol(mv::g_device_status, &zero, sizeof(zero));
    if (prev != device) cudaSetDevice(prev);
    return err == cudaSuccess ? MV_OK : cuda_fail(err, "clearing device status");
}

// Self-test of the failure path: one CTA waits on an mbarrier phase that
// nothing completes, with the kernels' bounded wait shortened to limit_ns;
// giving up raises the same sticky status bit a real wait would.
namespace mv {
__global__ void wait_timeout_selftest_kernel(unsigned long long limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) mbar_init(smem_addr(&bar), 1);
    fence_mbar_init();
    __syncthreads();
    const bool ok = mbar_wait_bounded_ns(smem_addr(&bar), 0, limit_ns);
    if (threadIdx.x == 0 && !ok) atomicOr(&g_device_status, kStatusWaitTimeout);
}
}  // namespace mv

int mv_selftest_wait_timeout(uint64_t limit_ns, void* stream) {
    if (limit_ns == 0 || limit_ns > 100000000ull)
        return fail(MV_ERR_INVALID_ARGUMENT, "limit_ns must be in (0, 100 ms]");
    mv::wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<unsigned long long>(limit_ns));
    const cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? MV_OK : cuda_fail(err, "self-test kernel launch");
}

// ------------------------------------------------- allocation-free decode

// Split-KV scratch of mv_paged_decode_noalloc: a file-scope device array, so
// callers that cannot allocate still get the split-KV kernels. Zero at module
// load; shared by every call on a device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[MV_NOALLOC_SCRATCH_BYTES];

int mv_paged_decode_noalloc(const void* q, int64_t q_stride_seq, int64_t q_stride_head,
                            const void* k_cache, const void* v_cache, int64_t num_blocks,
                            int32_t num_kv_heads, int32_t block_size, int32_t head_dim,
                            const void* block_table, int32_t block_table_type,
                            int64_t block_table_stride, int64_t blocks_per_seq,
                            const void* context_lens, int32_t context_lens_type,
                            int64_t max_context_len, int32_t batch, int32_t num_q_heads,
                            float scale, void* out, int64_t out_stride_seq,
                            int64_t out_stride_head, int32_t pages_per_split, uint32_t flags,
                            int32_t dtype, void* stream) {
    if (flags & MV_FLAG_FUSED_MERGE)
        return fail(MV_ERR_UNSUPPORTED,
                    "mv_paged_decode_noalloc does not take MV_FLAG_FUSED_MERGE (its counters must start at zero)");
    // The scratch the call's own plan needs: planned with the caches' real
    // alignment, as mv_paged_decode plans it (unaligned caches take the
    // CUDA-core kernel, whose split sizes differ).
    const Geometry g{batch, num_q_heads, num_kv_heads, head_dim, block_size, max_context_len, dtype};
    Plan plan;
    int rc = make_plan(g, pages_per_split, flags, tma_aligned(k_cache, v_cache), &plan, StreamUse::kAllowed);
    if (rc != MV_OK) return rc;
    const size_t needed = plan.workspace;
    if (needed > MV_NOALLOC_SCRATCH_BYTES)
        return fail(MV_ERR_UNSUPPORTED,
                    "mv_paged_decode_noalloc: this call needs %zu bytes of split-KV scratch, the "
                    "built-in array holds %zu; use mv_paged_decode with a workspace, or a larger "
                    "pages_per_split",
                    needed, static_cast<size_t>(MV_NOALLOC_SCRATCH_BYTES));
    // The array's name is a host-side stand-in: look up its device address,
    // with the call's device current. Outside stream capture every call looks
    // it up again (cheap), so a module reloaded after a cudaDeviceReset is
    // found at its new address; inside a capture the call uses the address its
    // device's last call outside capture found.
    static void* scratch[kMaxDevices] = {nullptr};
    static std::mutex scratch_mutex;
    int device = 0;
    cudaError_t err = cudaGetDevice(&device);
    if (err != cudaSuccess) return cuda_fail(err, "cudaGetDevice");
    if (device < 0 || device >= kMaxDevices) return fail(MV_ERR_UNSUPPORTED, "device index %d out of range", device);
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    err = cudaStreamIsCapturing(static_cast<cudaStream_t>(stream), &capture);
    if (err != cudaSuccess) return cuda_fail(err, "cudaStreamIsCapturing");
    void* ptr = nullptr;
    {
        std::lock_guard<std::mutex> lock(scratch_mutex);
        if (!scratch[device] || capture == cudaStreamCaptureStatusNone) {
            err = cudaGetSymbolAddress(&scratch[device], g_noalloc_scratch);
            if (err != cudaSuccess) {
                scratch[device] = nullptr;
                return cuda_fail(err, "cudaGetSymbolAddress of the no-alloc scratch");
            }
        }
        ptr = scratch[device];
    }
    return mv_paged_decode(q, q_stride_seq, q_stride_head, k_cache, v_cache, num_blocks, num_kv_heads,
                           block_size, head_dim, block_table, block_table_type, block_table_stride,
                           blocks_per_seq, context_lens, context_lens_type, max_context_len, batch,
                           num_q_heads, scale, out, out_stride_seq, out_stride_head, ptr,
                           MV_NOALLOC_SCRATCH_BYTES, pages_per_split, flags, dtype, stream);
}

}  // extern "C"
