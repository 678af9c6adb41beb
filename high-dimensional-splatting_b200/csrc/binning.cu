// binning.cu -- tile binning: pack + count, prefix sum, key emission, stable device radix sort,
// tile ranges.  Restates forward.cu:13-139 and 284-404 of the reference, replacing its thrust scan
// and CUB onesweep sort with this file's own kernels.
//
// The reference sorts one 64-bit key per (tile, gaussian) pair, tile << 32 | float bits of the
// depth, stably from gaussian order: every tile's list runs front to back, equal depths in gaussian
// order.  This file reaches the same order in two smaller sorts:
//   1. the gaussians that touch a tile are sorted stably by their 32 depth bits (4 passes over n
//      keys; gaussians that touch none get the largest key and sit, unused, at the end);
//   2. the pairs are emitted in that depth order and sorted stably by tile id alone (ceil(log2
//      tiles) bits, 2 passes for up to 65536 tiles, over the pairs).
// Stability carries the (depth, gaussian) order of step 1 into every tile's list.  Against a single
// 64-bit sort of the pairs this moves 4 n + 2 P keys instead of 6 P (P = pairs, about 3 n here).
//
// Each radix pass is (1) a per-block digit histogram, (2) an exclusive scan of the digit-major
// count table, (3) a stable scatter that ranks each key among equal digits of its block with
// __match_any_sync.  No inter-block waits, so nothing can spin.
#include "hds_common.cuh"

#include <climits>

namespace hds {
namespace {

constexpr int SCAN_THREADS = 512;
constexpr int SCAN_ITEMS = 8;
constexpr int SCAN_TILE = SCAN_THREADS * SCAN_ITEMS;  // 4096 items per block
constexpr int SORT_THREADS = 256;
constexpr int SORT_TILE = 4096;                        // keys per block and pass
constexpr int RADIX = 256;

inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// ---------------------------------------------------------------------------------------------
// exclusive scan (two levels: blocks of 4096, then one block over the block sums)
// ---------------------------------------------------------------------------------------------
template <typename T>
__device__ __forceinline__ T block_exclusive_scan(T v, T* s_warp, T& total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    T x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        T y = __shfl_up_sync(FULL_MASK, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[warp] = x;
    __syncthreads();
    if (warp == 0) {
        T w = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : T(0);
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            T y = __shfl_up_sync(FULL_MASK, w, o);
            if (lane >= o) w += y;
        }
        s_warp[lane] = w;  // inclusive warp totals
    }
    __syncthreads();
    T before = warp > 0 ? s_warp[warp - 1] : T(0);
    total = s_warp[(blockDim.x >> 5) - 1];
    __syncthreads();
    return before + x - v;
}

template <typename T>
__global__ void __launch_bounds__(SCAN_THREADS) scan_reduce_kernel(const T* __restrict__ in, int64_t n, T* __restrict__ block_sums) {
    __shared__ T s_warp[32];
    int64_t base = (int64_t)blockIdx.x * SCAN_TILE + (int64_t)threadIdx.x * SCAN_ITEMS;
    T sum = 0;
#pragma unroll
    for (int k = 0; k < SCAN_ITEMS; k++)
        if (base + k < n) sum += in[base + k];
    T total;
    block_exclusive_scan<T>(sum, s_warp, total);
    if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

template <typename T>
__global__ void __launch_bounds__(SCAN_THREADS) scan_block_sums_kernel(T* __restrict__ block_sums, int nblocks, T* __restrict__ total_out) {
    __shared__ T s_warp[32];
    int base = threadIdx.x * SCAN_ITEMS;
    T v[SCAN_ITEMS];
    T sum = 0;
#pragma unroll
    for (int k = 0; k < SCAN_ITEMS; k++) {
        v[k] = base + k < nblocks ? block_sums[base + k] : T(0);
        sum += v[k];
    }
    T total;
    T run = block_exclusive_scan<T>(sum, s_warp, total);
#pragma unroll
    for (int k = 0; k < SCAN_ITEMS; k++) {
        if (base + k < nblocks) block_sums[base + k] = run;
        run += v[k];
    }
    if (threadIdx.x == 0 && total_out) *total_out = total;
}

template <typename T>
__global__ void __launch_bounds__(SCAN_THREADS) scan_apply_kernel(const T* __restrict__ in, int64_t n, const T* __restrict__ block_sums,
                                                                  T* __restrict__ out) {
    __shared__ T s_warp[32];
    int64_t base = (int64_t)blockIdx.x * SCAN_TILE + (int64_t)threadIdx.x * SCAN_ITEMS;
    T v[SCAN_ITEMS];
    T sum = 0;
#pragma unroll
    for (int k = 0; k < SCAN_ITEMS; k++) {
        v[k] = base + k < n ? in[base + k] : T(0);
        sum += v[k];
    }
    T total;
    T run = block_exclusive_scan<T>(sum, s_warp, total) + block_sums[blockIdx.x];
#pragma unroll
    for (int k = 0; k < SCAN_ITEMS; k++) {
        if (base + k < n) out[base + k] = run;
        run += v[k];
    }
}

inline int64_t scan_blocks(int64_t n) { return (n + SCAN_TILE - 1) / SCAN_TILE; }

// Sum of n items into *total_out (device): the first two launches of exclusive_scan.
template <typename T>
int reduce_total(const T* in, int64_t n, T* block_sums, T* total_out, cudaStream_t stream) {
    int64_t nb = scan_blocks(n);
    HDS_REQUIRE(nb <= SCAN_TILE, HDS_ERR_TOO_LARGE, "sum of %lld items exceeds %d", (long long)n, SCAN_TILE * SCAN_TILE);
    if (n == 0) {
        HDS_CHECK_CUDA(cudaMemsetAsync(total_out, 0, sizeof(T), stream));
        return HDS_OK;
    }
    scan_reduce_kernel<T><<<(unsigned)nb, SCAN_THREADS, 0, stream>>>(in, n, block_sums);
    scan_block_sums_kernel<T><<<1, SCAN_THREADS, 0, stream>>>(block_sums, (int)nb, total_out);
    note_launches(1);
    HDS_CHECK_LAUNCH("reduce_total");
    return HDS_OK;
}

// Exclusive scan of n items; block_sums holds scan_blocks(n) entries; *total_out (device) gets the sum.
template <typename T>
int exclusive_scan(const T* in, T* out, int64_t n, T* block_sums, T* total_out, cudaStream_t stream) {
    int64_t nb = scan_blocks(n);
    HDS_REQUIRE(nb <= SCAN_TILE, HDS_ERR_TOO_LARGE, "scan of %lld items exceeds %d", (long long)n, SCAN_TILE * SCAN_TILE);
    if (n == 0) {
        if (total_out) HDS_CHECK_CUDA(cudaMemsetAsync(total_out, 0, sizeof(T), stream));
        return HDS_OK;
    }
    scan_reduce_kernel<T><<<(unsigned)nb, SCAN_THREADS, 0, stream>>>(in, n, block_sums);
    scan_block_sums_kernel<T><<<1, SCAN_THREADS, 0, stream>>>(block_sums, (int)nb, total_out);
    scan_apply_kernel<T><<<(unsigned)nb, SCAN_THREADS, 0, stream>>>(in, n, block_sums, out);
    note_launches(2);  // the reduce and block-sum launches; HDS_CHECK_LAUNCH counts the third
    HDS_CHECK_LAUNCH("exclusive_scan");
    return HDS_OK;
}

// ---------------------------------------------------------------------------------------------
// pack + count (forward.cu:13-61)
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) prepare_kernel(int n, const float2* __restrict__ means2D, const float* __restrict__ depths,
                                                      const float* __restrict__ radii, const float* __restrict__ conics,
                                                      const float* __restrict__ colors, const float* __restrict__ opacities,
                                                      int tiles_x, int row0, int tiles_y, float4* __restrict__ conic4,
                                                      float4* __restrict__ color_opacity, int4* __restrict__ rect,
                                                      int64_t* __restrict__ touched) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float a = conics[3 * i], b = conics[3 * i + 1], c = conics[3 * i + 2];
    float o = opacities[i];
    conic4[i] = make_float4(a, b, c, 0.0f);
    color_opacity[i] = make_float4(colors[3 * i], colors[3 * i + 1], colors[3 * i + 2], o);
    int x0 = 0, y0 = 0, x1 = -1, y1 = -1;
    int count = 0;
    float2 m = means2D[i];
    // Written as radius > 0 so a NaN radius is culled too (forward.cu:31-36).
    if (radii[i] > 0.0f && tile_rect(m.x, m.y, a, b, c, o, tiles_x, row0, tiles_y, x0, y0, x1, y1))
        count = (x1 - x0 + 1) * (y1 - y0 + 1);
    rect[i] = make_int4(x0, y0, x1 - x0 + 1, (int)__float_as_uint(depths[i]));
    touched[i] = count;
}

// ---------------------------------------------------------------------------------------------
// depth sort of the gaussians, then pair emission in depth order (forward.cu:63-113)
// ---------------------------------------------------------------------------------------------
constexpr uint32_t NO_TILES_KEY = 0xffffffffu;

__global__ void __launch_bounds__(256) gaussian_keys_kernel(int n, const int4* __restrict__ rect,
                                                            const int64_t* __restrict__ touched,
                                                            uint32_t* __restrict__ keys, int32_t* __restrict__ values) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    keys[i] = touched[i] > 0 ? (uint32_t)rect[i].w : NO_TILES_KEY;
    values[i] = i;
}

// Pair counts in depth order, for the scan that places each gaussian's pairs.
__global__ void __launch_bounds__(256) sorted_counts_kernel(int n, const int32_t* __restrict__ order,
                                                            const int64_t* __restrict__ touched,
                                                            int64_t* __restrict__ counts) {
    int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j < n) counts[j] = touched[order[j]];
}

// Largest j in [lo, hi] with offsets[j] <= o: the owner of pair o (gaussians without pairs share
// their successor's offset and are skipped).
template <typename T>
__device__ __forceinline__ int owner_of(const T* offsets, int lo, int hi, int64_t o) {
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (offsets[mid] <= o) lo = mid; else hi = mid - 1;
    }
    return lo;
}

constexpr int EMIT_THREADS = 256;
constexpr int EMIT_TILE = 2048;  // pairs per block

// One block per 2048 consecutive pairs: the owners of its first and last pair bound the gaussians it
// needs, whose offsets it stages in shared memory and searches there.  Every gaussian strictly
// between two owners has at least one pair, so a block spans at most 2048 gaussians; a longer span
// (which would need pairless gaussians among the pair owners) searches global memory instead.
__global__ void __launch_bounds__(EMIT_THREADS) emit_kernel(int64_t total, int n, const int64_t* __restrict__ offsets,
                                                            const int32_t* __restrict__ order,
                                                            const int4* __restrict__ rect, int tiles_x,
                                                            uint32_t* __restrict__ tile_keys,
                                                            int32_t* __restrict__ values) {
    __shared__ int64_t s_off[EMIT_TILE];
    __shared__ int s_owner[2];
    const int64_t o0 = (int64_t)blockIdx.x * EMIT_TILE;
    const int64_t o1 = min(total, o0 + EMIT_TILE);
    if (threadIdx.x < 2) s_owner[threadIdx.x] = owner_of(offsets, 0, n - 1, threadIdx.x == 0 ? o0 : o1 - 1);
    __syncthreads();
    const int j0 = s_owner[0], span = s_owner[1] - j0 + 1;
    const bool staged = span <= EMIT_TILE;
    if (staged)
        for (int t = threadIdx.x; t < span; t += EMIT_THREADS) s_off[t] = offsets[j0 + t];
    __syncthreads();
    for (int64_t o = o0 + threadIdx.x; o < o1; o += EMIT_THREADS) {
        int j;
        int64_t start;
        if (staged) {
            const int r = owner_of(s_off, 0, span - 1, o);
            j = j0 + r;
            start = s_off[r];
        } else {
            j = owner_of(offsets, j0, j0 + span - 1, o);
            start = offsets[j];
        }
        const int g = order[j];
        const int4 r = rect[g];
        const int local = (int)(o - start);
        const int tx = r.x + local % r.z, ty = r.y + local / r.z;
        tile_keys[o] = (uint32_t)(ty * tiles_x + tx);
        values[o] = g;
    }
}

// ---------------------------------------------------------------------------------------------
// radix sort passes (32-bit keys)
// ---------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(SORT_THREADS) radix_histogram_kernel(const uint32_t* __restrict__ keys, int64_t n,
                                                                       int shift, uint32_t* __restrict__ counts,
                                                                       int nblocks) {
    __shared__ uint32_t hist[RADIX];
    hist[threadIdx.x] = 0;
    __syncthreads();
    int64_t begin = (int64_t)blockIdx.x * SORT_TILE;
    int64_t end = min(n, begin + SORT_TILE);
    const int lane = threadIdx.x & 31;
    for (int64_t r = begin; r < end; r += SORT_THREADS) {
        int64_t i = r + threadIdx.x;
        uint32_t d = i < end ? (keys[i] >> shift) & (RADIX - 1) : RADIX;
        // Warp-aggregated: one shared atomic per distinct digit of the warp.
        uint32_t peers = __match_any_sync(FULL_MASK, d);
        if (d < RADIX && lane == __ffs(peers) - 1) atomicAdd(&hist[d], __popc(peers));
    }
    __syncthreads();
    counts[threadIdx.x * nblocks + blockIdx.x] = hist[threadIdx.x];
}

__global__ void __launch_bounds__(SORT_THREADS) radix_scatter_kernel(const uint32_t* __restrict__ keys_in,
                                                                     const int32_t* __restrict__ vals_in, int64_t n,
                                                                     int shift, const uint32_t* __restrict__ offsets,
                                                                     int nblocks, uint32_t* __restrict__ keys_out,
                                                                     int32_t* __restrict__ vals_out) {
    constexpr int WARPS = SORT_THREADS / 32;
    __shared__ uint32_t s_base[RADIX];
    __shared__ uint32_t s_warp[WARPS][RADIX];
    __shared__ uint32_t s_total[RADIX];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t begin = (int64_t)blockIdx.x * SORT_TILE;
    const int64_t end = min(n, begin + SORT_TILE);
    s_base[tid] = offsets[tid * nblocks + blockIdx.x];
    for (int64_t r = begin; r < end; r += SORT_THREADS) {
#pragma unroll
        for (int w = 0; w < WARPS; w++) s_warp[w][tid] = 0;
        __syncthreads();
        int64_t i = r + tid;
        bool valid = i < end;
        uint32_t key = valid ? keys_in[i] : 0;
        int32_t val = valid ? vals_in[i] : 0;
        uint32_t d = valid ? (key >> shift) & (RADIX - 1) : RADIX;
        uint32_t peers = __match_any_sync(FULL_MASK, d);
        uint32_t rank = __popc(peers & ((1u << lane) - 1u));
        if (valid && lane == __ffs(peers) - 1) s_warp[warp][d] = __popc(peers);
        __syncthreads();
        uint32_t run = 0;
#pragma unroll
        for (int w = 0; w < WARPS; w++) {
            uint32_t c = s_warp[w][tid];
            s_warp[w][tid] = run;
            run += c;
        }
        s_total[tid] = run;
        __syncthreads();
        if (valid) {
            uint32_t pos = s_base[d] + s_warp[warp][d] + rank;
            keys_out[pos] = key;
            vals_out[pos] = val;
        }
        __syncthreads();
        s_base[tid] += s_total[tid];
    }
}

int sort_blocks(int64_t n) { return (int)((n + SORT_TILE - 1) / SORT_TILE); }

// Stable LSD sort of (key, value) pairs on bits [0, 8 passes): ping-pongs between the a and b
// buffers, so the result is in a after an even number of passes and in b after an odd one.
int radix_sort(uint32_t* keys_a, uint32_t* keys_b, int32_t* vals_a, int32_t* vals_b, int64_t n, int passes,
               uint32_t* counts, uint32_t* count_sums, cudaStream_t stream) {
    const int nblocks = sort_blocks(n);
    const int64_t table = (int64_t)RADIX * nblocks;
    for (int p = 0; p < passes; p++) {
        radix_histogram_kernel<<<nblocks, SORT_THREADS, 0, stream>>>(keys_a, n, 8 * p, counts, nblocks);
        HDS_CHECK_LAUNCH("radix_histogram_kernel");
        if (int rc = exclusive_scan<uint32_t>(counts, counts, table, count_sums, nullptr, stream)) return rc;
        radix_scatter_kernel<<<nblocks, SORT_THREADS, 0, stream>>>(keys_a, vals_a, n, 8 * p, counts, nblocks, keys_b,
                                                                   vals_b);
        HDS_CHECK_LAUNCH("radix_scatter_kernel");
        uint32_t* tk = keys_a; keys_a = keys_b; keys_b = tk;
        int32_t* tv = vals_a; vals_a = vals_b; vals_b = tv;
    }
    return HDS_OK;
}

__global__ void __launch_bounds__(256) tile_ranges_kernel(int64_t total, const uint32_t* __restrict__ tile_keys,
                                                          int2* __restrict__ ranges) {
    int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= total) return;
    uint32_t tile = tile_keys[k];
    if (k == 0 || tile_keys[k - 1] != tile) ranges[tile].x = (int)k;
    if (k == total - 1 || tile_keys[k + 1] != tile) ranges[tile].y = (int)(k + 1);
}

// The reference's 64-bit keys of the sorted pairs, tile << 32 | depth bits, for callers that ask.
__global__ void __launch_bounds__(256) full_keys_kernel(int64_t total, const uint32_t* __restrict__ tile_keys,
                                                        const int32_t* __restrict__ values,
                                                        const int4* __restrict__ rect, uint64_t* __restrict__ keys) {
    int64_t k = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (k < total) keys[k] = ((uint64_t)tile_keys[k] << 32) | (uint32_t)rect[values[k]].w;
}

// Scratch layouts --------------------------------------------------------------------------------
struct PrepareLayout {
    size_t rect, touched, block_sums, total, bytes;
    explicit PrepareLayout(int n) {
        size_t nn = (size_t)(n > 0 ? n : 1);
        rect = 0;
        touched = rect + align256(nn * sizeof(int4));
        block_sums = touched + align256(nn * sizeof(int64_t));
        total = block_sums + align256((size_t)scan_blocks((int64_t)nn) * sizeof(int64_t));
        bytes = total + 256;
    }
};

int tile_bits_for(int tiles) {
    int bits = 0;
    while ((1 << bits) < tiles) bits++;
    return bits;
}

struct SortLayout {
    // Gaussian depth sort: keys and values in two buffers each, then the depth-ordered pair counts and
    // their offsets.  Pair sort: tile keys in two buffers, values in values_sorted and one more.
    size_t g_keys_a, g_keys_b, g_vals_a, g_vals_b, g_counts, g_offsets, g_block_sums;
    size_t p_keys_a, p_keys_b, p_vals_other, counts, count_sums, bytes;
    int pair_passes;
    SortLayout(int n, int64_t dups, int tiles) {
        const size_t nn = (size_t)(n > 0 ? n : 1), d = (size_t)(dups > 0 ? dups : 1);
        pair_passes = (tile_bits_for(tiles) + 7) / 8;
        g_keys_a = 0;
        g_keys_b = g_keys_a + align256(nn * sizeof(uint32_t));
        g_vals_a = g_keys_b + align256(nn * sizeof(uint32_t));
        g_vals_b = g_vals_a + align256(nn * sizeof(int32_t));
        g_counts = g_vals_b + align256(nn * sizeof(int32_t));
        g_offsets = g_counts + align256(nn * sizeof(int64_t));
        g_block_sums = g_offsets + align256(nn * sizeof(int64_t));
        p_keys_a = g_block_sums + align256((size_t)scan_blocks((int64_t)nn) * sizeof(int64_t));
        p_keys_b = p_keys_a + align256(d * sizeof(uint32_t));
        p_vals_other = p_keys_b + align256(d * sizeof(uint32_t));
        counts = p_vals_other + align256(d * sizeof(int32_t));
        const size_t table = (size_t)RADIX * (size_t)max(sort_blocks((int64_t)nn), sort_blocks((int64_t)d));
        count_sums = counts + align256(table * sizeof(uint32_t));
        bytes = count_sums + align256((size_t)scan_blocks((int64_t)table) * sizeof(uint32_t)) + 256;
    }
};

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" size_t hds_rasterize_prepare_scratch_bytes(int n) { return PrepareLayout(n).bytes; }

extern "C" int hds_rasterize_prepare(int n, const float* means2D, const float* depths, const float* radii,
                                     const float* conics, const float* colors, const float* opacities, int width,
                                     int height, int origin_y, float* conic4, float* color_opacity, void* scratch,
                                     size_t scratch_bytes, int64_t* num_duplicates, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0 && num_duplicates, HDS_ERR_INVALID,
                "rasterize: bad arguments (n=%d, %dx%d)", n, width, height);
    HDS_REQUIRE(origin_y >= 0 && origin_y % TILE == 0, HDS_ERR_INVALID,
                "rasterize: origin_y %d must be a non-negative multiple of 16", origin_y);
    PrepareLayout L(n);
    HDS_REQUIRE(scratch && scratch_bytes >= L.bytes, HDS_ERR_SCRATCH, "rasterize: prepare scratch needs %zu bytes",
                L.bytes);
    HDS_REQUIRE(((uintptr_t)scratch & 255) == 0 && ((uintptr_t)conic4 & 15) == 0 && ((uintptr_t)color_opacity & 15) == 0 &&
                    ((uintptr_t)means2D & 7) == 0,
                HDS_ERR_INVALID, "rasterize: scratch must be 256-byte, conic/color_opacity 16-byte aligned");
    *num_duplicates = 0;
    if (n == 0) return HDS_OK;
    char* s = static_cast<char*>(scratch);
    auto* rect = reinterpret_cast<int4*>(s + L.rect);
    auto* touched = reinterpret_cast<int64_t*>(s + L.touched);
    auto* block_sums = reinterpret_cast<int64_t*>(s + L.block_sums);
    auto* total = reinterpret_cast<int64_t*>(s + L.total);
    int tx = tiles_for(width), ty = tiles_for(height);
    prepare_kernel<<<(n + 255) / 256, 256, 0, stream>>>(n, reinterpret_cast<const float2*>(means2D), depths, radii, conics,
                                                        colors, opacities, tx, origin_y / TILE, ty,
                                                        reinterpret_cast<float4*>(conic4),
                                                        reinterpret_cast<float4*>(color_opacity), rect, touched);
    HDS_CHECK_LAUNCH("prepare_kernel");
    if (int rc = reduce_total<int64_t>(touched, n, block_sums, total, stream)) return rc;
    int64_t host_total = 0;
    HDS_CHECK_CUDA(cudaMemcpyAsync(&host_total, total, sizeof(int64_t), cudaMemcpyDeviceToHost, stream));
    HDS_CHECK_CUDA(cudaStreamSynchronize(stream));
    HDS_REQUIRE(host_total <= INT_MAX, HDS_ERR_TOO_LARGE,
                "rasterize: %lld (tile, gaussian) pairs overflow the int32 tile ranges", (long long)host_total);
    *num_duplicates = host_total;
    return HDS_OK;
}

extern "C" size_t hds_rasterize_sort_scratch_bytes(int n, int64_t num_duplicates, int width, int height) {
    return SortLayout(n, num_duplicates, tiles_for(width) * tiles_for(height)).bytes;
}

extern "C" int hds_rasterize_sort(int n, int64_t num_duplicates, int width, int height, const void* prepare_scratch,
                                  void* scratch, size_t scratch_bytes, int32_t* values_sorted, int32_t* tile_ranges,
                                  uint64_t* keys_sorted, hds_stream_t stream) {
    clear_error();
    int tiles = tiles_for(width) * tiles_for(height);
    HDS_REQUIRE(n > 0 && num_duplicates > 0 && num_duplicates <= INT_MAX && width > 0 && height > 0, HDS_ERR_INVALID,
                "rasterize: bad sort arguments (n=%d, pairs=%lld)", n, (long long)num_duplicates);
    SortLayout L(n, num_duplicates, tiles);
    HDS_REQUIRE(scratch && scratch_bytes >= L.bytes && ((uintptr_t)scratch & 255) == 0, HDS_ERR_SCRATCH,
                "rasterize: sort scratch needs %zu bytes, 256-byte aligned", L.bytes);
    PrepareLayout P(n);
    const char* ps = static_cast<const char*>(prepare_scratch);
    const auto* rect = reinterpret_cast<const int4*>(ps + P.rect);
    const auto* touched = reinterpret_cast<const int64_t*>(ps + P.touched);
    char* s = static_cast<char*>(scratch);
    auto* counts = reinterpret_cast<uint32_t*>(s + L.counts);
    auto* count_sums = reinterpret_cast<uint32_t*>(s + L.count_sums);

    // 1. Gaussians by depth (4 passes: the result is back in the a buffers).
    auto* g_keys_a = reinterpret_cast<uint32_t*>(s + L.g_keys_a);
    auto* g_vals_a = reinterpret_cast<int32_t*>(s + L.g_vals_a);
    gaussian_keys_kernel<<<(n + 255) / 256, 256, 0, stream>>>(n, rect, touched, g_keys_a, g_vals_a);
    HDS_CHECK_LAUNCH("gaussian_keys_kernel");
    if (int rc = radix_sort(g_keys_a, reinterpret_cast<uint32_t*>(s + L.g_keys_b), g_vals_a,
                            reinterpret_cast<int32_t*>(s + L.g_vals_b), n, 4, counts, count_sums, stream))
        return rc;
    const int32_t* order = g_vals_a;
    auto* g_counts = reinterpret_cast<int64_t*>(s + L.g_counts);
    auto* g_offsets = reinterpret_cast<int64_t*>(s + L.g_offsets);
    sorted_counts_kernel<<<(n + 255) / 256, 256, 0, stream>>>(n, order, touched, g_counts);
    HDS_CHECK_LAUNCH("sorted_counts_kernel");
    if (int rc = exclusive_scan<int64_t>(g_counts, g_offsets, n, reinterpret_cast<int64_t*>(s + L.g_block_sums),
                                         nullptr, stream))
        return rc;

    // 2. Pairs in depth order, then stably by tile.  The last pass must land in values_sorted: with an
    // even number of passes the emission buffer is values_sorted itself, with an odd one the scratch one.
    const int64_t total = num_duplicates;
    int32_t* vals_other = reinterpret_cast<int32_t*>(s + L.p_vals_other);
    int32_t* vals_a = (L.pair_passes % 2 == 0) ? values_sorted : vals_other;
    int32_t* vals_b = (L.pair_passes % 2 == 0) ? vals_other : values_sorted;
    auto* keys_a = reinterpret_cast<uint32_t*>(s + L.p_keys_a);
    auto* keys_b = reinterpret_cast<uint32_t*>(s + L.p_keys_b);
    emit_kernel<<<(unsigned)((total + EMIT_TILE - 1) / EMIT_TILE), EMIT_THREADS, 0, stream>>>(
        total, n, g_offsets, order, rect, tiles_for(width), keys_a, vals_a);
    HDS_CHECK_LAUNCH("emit_kernel");
    if (int rc = radix_sort(keys_a, keys_b, vals_a, vals_b, total, L.pair_passes, counts, count_sums, stream))
        return rc;
    const uint32_t* tile_keys = (L.pair_passes % 2 == 0) ? keys_a : keys_b;

    const unsigned blocks = (unsigned)((total + 255) / 256);
    HDS_CHECK_CUDA(cudaMemsetAsync(tile_ranges, 0, sizeof(int32_t) * 2 * (size_t)tiles, stream));
    tile_ranges_kernel<<<blocks, 256, 0, stream>>>(total, tile_keys, reinterpret_cast<int2*>(tile_ranges));
    HDS_CHECK_LAUNCH("tile_ranges_kernel");
    if (keys_sorted) {
        full_keys_kernel<<<blocks, 256, 0, stream>>>(total, tile_keys, values_sorted, rect, keys_sorted);
        HDS_CHECK_LAUNCH("full_keys_kernel");
    }
    return HDS_OK;
}
