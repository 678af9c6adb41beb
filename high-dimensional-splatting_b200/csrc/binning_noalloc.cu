// binning_noalloc.cu -- tile binning for callers that cannot allocate device memory.
//
// Some callers cannot allocate device memory at the point where they bin a frame.  Examples:
//   * a renderer embedded in a host application whose GPU memory belongs to another allocator;
//   * a real-time loop that may not call cudaMalloc, because cudaMalloc can synchronise the
//     device and stall the frame;
//   * an FFI caller (Go, Java, ...) that only holds buffers handed to it by its host.
// hds_rasterize_prepare and hds_rasterize_sort need caller-provided scratch sized per call.  This
// file gives such callers hds_rasterize_bin_noalloc instead.  It runs the same two steps on the same
// kernels, with their scratch in one file-scope device array of HDS_NOALLOC_SCRATCH_BYTES (64 MiB).
//
// The array lives in this file's own module, so only processes that call this entry point pay for
// it; once loaded, every GPU that used it holds the 64 MiB until the process exits.  Host code
// reaches it only through the address cudaGetSymbolAddress returns (the symbol's name is a
// host-side stand-in, not a device address).  That address is looked up once per device, on the
// first call made with that device current.
#include <mutex>

#include "hds_common.cuh"

namespace hds {
namespace {

constexpr size_t kScratchBytes = HDS_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_bin_scratch[kScratchBytes];

std::mutex g_mutex;
void* g_scratch_address[kMaxDevices] = {};

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Device address of g_bin_scratch for the current device (set-up on the first call per device).
int scratch_address(void** out) {
    int dev = -1;
    HDS_CHECK_CUDA(cudaGetDevice(&dev));
    HDS_REQUIRE(dev >= 0 && dev < kMaxDevices, HDS_ERR_INVALID, "rasterize_bin_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_mutex);
    if (g_scratch_address[dev] == nullptr) {
        void* p = nullptr;
        cudaError_t err = cudaGetSymbolAddress(&p, g_bin_scratch);
        if (err != cudaSuccess) return cuda_fail(err, "cudaGetSymbolAddress(g_bin_scratch)");
        g_scratch_address[dev] = p;
    }
    *out = g_scratch_address[dev];
    return HDS_OK;
}

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" int hds_rasterize_bin_noalloc(int n, const float* means2D, const float* depths, const float* radii,
                                         const float* conics, const float* colors, const float* opacities, int width,
                                         int height, float* conic4, float* color_opacity, int32_t* values_sorted,
                                         int64_t values_capacity, int32_t* tile_ranges, int64_t* num_duplicates,
                                         hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0 && num_duplicates && tile_ranges, HDS_ERR_INVALID,
                "rasterize_bin_noalloc: bad arguments (n=%d, %dx%d)", n, width, height);
    const size_t prep = align256(hds_rasterize_prepare_scratch_bytes(n));
    HDS_REQUIRE(prep <= kScratchBytes, HDS_ERR_TOO_LARGE,
                "rasterize_bin_noalloc: %d gaussians need %zu bytes of scratch, more than the fixed %zu", n, prep,
                kScratchBytes);
    void* base = nullptr;
    if (int rc = scratch_address(&base)) return rc;
    char* scratch = static_cast<char*>(base);

    // Step 1 (pack, count, scan, host read of the pair count) into the front of the array.
    if (int rc = hds_rasterize_prepare(n, means2D, depths, radii, conics, colors, opacities, width, height, 0, conic4,
                                       color_opacity, scratch, prep, num_duplicates, stream))
        return rc;
    const int64_t dups = *num_duplicates;
    const int tiles = tiles_for(width) * tiles_for(height);
    if (dups == 0) {
        HDS_CHECK_CUDA(cudaMemsetAsync(tile_ranges, 0, sizeof(int32_t) * 2 * (size_t)tiles, stream));
        return HDS_OK;
    }
    HDS_REQUIRE(dups <= values_capacity, HDS_ERR_TOO_LARGE,
                "rasterize_bin_noalloc: %lld (tile, gaussian) pairs exceed values_sorted capacity %lld", (long long)dups,
                (long long)values_capacity);
    const size_t sort = hds_rasterize_sort_scratch_bytes(n, dups, width, height);
    HDS_REQUIRE(prep + sort <= kScratchBytes, HDS_ERR_TOO_LARGE,
                "rasterize_bin_noalloc: %d gaussians with %lld pairs need %zu bytes of scratch, more than the fixed %zu",
                n, (long long)dups, prep + sort, kScratchBytes);
    // Step 2 (emit, radix sort, tile ranges) behind it.  Every scratch byte either step reads was
    // written earlier in this same call, so nothing left by a previous call needs clearing; the tile
    // ranges (an output) are zeroed by the sort step itself.
    return hds_rasterize_sort(n, dups, width, height, scratch, scratch + prep, sort, values_sorted, tile_ranges,
                              nullptr, stream);
}
