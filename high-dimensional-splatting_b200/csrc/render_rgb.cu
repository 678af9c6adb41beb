// render_rgb.cu -- front-to-back FP32 RGB blend over the sorted tile lists, and its backward.
//
// Restates forward.cu:141-237 (render_gaussians) and backward.cu:7-164 (render_gaussians_backward)
// of the reference.  One block per 16x16 tile; the tile's list is staged through shared memory in
// batches of 256 entries.  Each warp owns an 8x4 pixel block and skips the gaussians whose
// opacity-aware box misses it.  The per-pair arithmetic is pair_alpha() and the blend update below, in
// the same order as the CPU oracle, so image, final_T and n_contrib are bit-identical to it.
#include "hds_common.cuh"

namespace hds {
namespace {

constexpr int BATCH = TILE_PIXELS;

// Pixel of thread tid inside its 16x16 tile: warp w owns the 8x4 block at ((w & 1) * 8, (w >> 1) * 4), so
// a warp's pixels are compact and one box test decides whether a gaussian can touch any of them.
__device__ __forceinline__ int2 tile_pixel(int tid) {
    const int warp = tid >> 5, lane = tid & 31;
    return make_int2((warp & 1) * 8 + (lane & 7), (warp >> 1) * 4 + (lane >> 3));
}

__global__ void __launch_bounds__(TILE_PIXELS) rgb_forward_kernel(int width, int height, int tiles_x, int origin_y,
                                                                  const int2* __restrict__ ranges,
                                                                  const int32_t* __restrict__ values,
                                                                  const float2* __restrict__ means2D,
                                                                  const float4* __restrict__ conic4,
                                                                  const float4* __restrict__ color_opacity,
                                                                  const float* __restrict__ background,
                                                                  float4* __restrict__ image4, float* __restrict__ final_T,
                                                                  int32_t* __restrict__ n_contrib) {
    __shared__ float2 s_mean[BATCH];
    __shared__ float4 s_conic[BATCH];
    __shared__ float4 s_color[BATCH];
    __shared__ float2 s_ext[BATCH];
    const int tid = threadIdx.x, warp = tid >> 5;
    const int tile = blockIdx.x;
    const int x0 = (tile % tiles_x) * TILE, y0 = (tile / tiles_x) * TILE;
    const int2 lp = tile_pixel(tid);
    const int px = x0 + lp.x, py = y0 + lp.y;
    const bool inside = px < width && py < height;
    const float cx = (float)px + 0.5f, cy = (float)(py + origin_y) + 0.5f;
    const float wx0 = (float)(x0 + (warp & 1) * 8) + 0.5f, wx1 = wx0 + 7.0f;
    const float wy0 = (float)(y0 + origin_y + (warp >> 1) * 4) + 0.5f, wy1 = wy0 + 3.0f;
    const int2 range = ranges[tile];
    const int count = range.y - range.x;

    float T = 1.0f;
    float ar = 0.0f, ag = 0.0f, ab = 0.0f;
    int last = 0;
    bool done = !inside;
    for (int base = 0; base < count; base += BATCH) {
        // Also the barrier that protects the previous batch's shared reads.
        if (__syncthreads_count(!done) == 0) break;
        int j = base + tid;
        if (j < count) {
            int g = values[range.x + j];
            float4 q = conic4[g], col = color_opacity[g];
            s_mean[tid] = means2D[g];
            s_conic[tid] = q;
            s_color[tid] = col;
            s_ext[tid] = cull_extent(q.x, q.y, q.z, col.w);
        }
        __syncthreads();
        const int n = min(BATCH, count - base);
        for (int k = 0; k < n && !done; k++) {
            float2 m = s_mean[k];
            // Warp-uniform: a gaussian whose box misses this warp's pixels has alpha < MIN_ALPHA on all of them.
            if (!box_hits(m, s_ext[k], wx0, wx1, wy0, wy1)) continue;
            float4 q = s_conic[k];
            float4 col = s_color[k];
            PairAlpha pa = pair_alpha(cx, cy, m.x, m.y, q.x, q.y, q.z, col.w);
            float alpha = fminf(MAX_ALPHA, pa.raw);
            if (alpha < MIN_ALPHA) continue;
            float test = T * (1.0f - alpha);
            if (test < MIN_T) {
                done = true;
                break;
            }
            float w = alpha * T;
            ar = fmaf(w, col.x, ar);
            ag = fmaf(w, col.y, ag);
            ab = fmaf(w, col.z, ab);
            T = test;
            last = base + k + 1;
        }
    }
    if (inside) {
        int p = py * width + px;
        image4[p] = make_float4(fmaf(T, background[0], ar), fmaf(T, background[1], ag), fmaf(T, background[2], ab), 0.0f);
        final_T[p] = T;
        n_contrib[p] = last;
    }
}

// Sums 8 values over a warp, scattered: afterwards lane l holds the total of value (l >> 2) & 7.
__device__ __forceinline__ float warp_reduce_scatter8(float v[8], int lane) {
    // 8 -> 4
    {
        bool hi = lane & 16;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float send = hi ? v[i] : v[i + 4];
            float keep = hi ? v[i + 4] : v[i];
            v[i] = keep + __shfl_xor_sync(FULL_MASK, send, 16);
        }
    }
    // 4 -> 2
    {
        bool hi = lane & 8;
#pragma unroll
        for (int i = 0; i < 2; i++) {
            float send = hi ? v[i] : v[i + 2];
            float keep = hi ? v[i + 2] : v[i];
            v[i] = keep + __shfl_xor_sync(FULL_MASK, send, 8);
        }
    }
    // 2 -> 1
    {
        bool hi = lane & 4;
        float send = hi ? v[0] : v[1];
        float keep = hi ? v[1] : v[0];
        v[0] = keep + __shfl_xor_sync(FULL_MASK, send, 4);
    }
    v[0] += __shfl_xor_sync(FULL_MASK, v[0], 2);
    v[0] += __shfl_xor_sync(FULL_MASK, v[0], 1);
    return v[0];
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(FULL_MASK, x, o);
    return x;
}

__global__ void __launch_bounds__(TILE_PIXELS) rgb_backward_kernel(
    int width, int height, int tiles_x, int origin_y, const int2* __restrict__ ranges, const int32_t* __restrict__ values,
    const float2* __restrict__ means2D, const float4* __restrict__ conic4, const float4* __restrict__ color_opacity,
    const float* __restrict__ background, const float* __restrict__ final_T_in, const int32_t* __restrict__ n_contrib,
    const float* __restrict__ grad_image, float* __restrict__ grad_means2D, float* __restrict__ grad_conics,
    float* __restrict__ grad_colors, float* __restrict__ grad_opacities) {
    __shared__ int s_id[BATCH];
    __shared__ float2 s_mean[BATCH];
    __shared__ float4 s_conic[BATCH];
    __shared__ float4 s_color[BATCH];
    __shared__ float2 s_ext[BATCH];
    __shared__ int s_max_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tile = blockIdx.x;
    const int x0 = (tile % tiles_x) * TILE, y0 = (tile / tiles_x) * TILE;
    const int2 lp = tile_pixel(tid);
    const int px = x0 + lp.x, py = y0 + lp.y;
    const float wx0 = (float)(x0 + (warp & 1) * 8) + 0.5f, wx1 = wx0 + 7.0f;
    const float wy0 = (float)(y0 + origin_y + (warp >> 1) * 4) + 0.5f, wy1 = wy0 + 3.0f;
    const bool inside = px < width && py < height;
    const float cx = (float)px + 0.5f, cy = (float)(py + origin_y) + 0.5f;
    const int2 range = ranges[tile];
    const int p = py * width + px;

    float T = inside ? final_T_in[p] : 0.0f;
    const float fT = T;
    const int last = inside ? n_contrib[p] : 0;
    float gp0 = 0.0f, gp1 = 0.0f, gp2 = 0.0f;
    if (inside) {
        gp0 = grad_image[3 * p];
        gp1 = grad_image[3 * p + 1];
        gp2 = grad_image[3 * p + 2];
    }
    const float dL_dfinal = background[0] * gp0 + background[1] * gp1 + background[2] * gp2;

    if (tid == 0) s_max_last = 0;
    __syncthreads();
    atomicMax(&s_max_last, last);
    __syncthreads();
    const int todo = min(range.y - range.x, s_max_last);

    float acc0 = 0.0f, acc1 = 0.0f, acc2 = 0.0f;
    float lc0 = 0.0f, lc1 = 0.0f, lc2 = 0.0f, last_alpha = 0.0f;
    for (int end = todo; end > 0; end -= BATCH) {
        const int n = min(BATCH, end);
        const int start = end - n;
        __syncthreads();
        if (tid < n) {
            int g = values[range.x + start + tid];
            float4 q = conic4[g], col = color_opacity[g];
            s_id[tid] = g;
            s_mean[tid] = means2D[g];
            s_conic[tid] = q;
            s_color[tid] = col;
            s_ext[tid] = cull_extent(q.x, q.y, q.z, col.w);
        }
        __syncthreads();
        for (int k = n - 1; k >= 0; k--) {
            // Warp-uniform skip of gaussians whose box misses this warp's pixels (they never blended there).
            if (!box_hits(s_mean[k], s_ext[k], wx0, wx1, wy0, wy1)) continue;
            float v[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
            float v8 = 0.0f;
            bool contributes = inside && start + k < last;
            if (contributes) {
                float2 m = s_mean[k];
                float4 q = s_conic[k];
                float4 col = s_color[k];
                PairAlpha pa = pair_alpha(cx, cy, m.x, m.y, q.x, q.y, q.z, col.w);
                float alpha = fminf(MAX_ALPHA, pa.raw);
                contributes = alpha >= MIN_ALPHA;
                if (contributes) {
                    float one_m = 1.0f - alpha;
                    T = T / one_m;
                    acc0 = last_alpha * lc0 + (1.0f - last_alpha) * acc0;
                    acc1 = last_alpha * lc1 + (1.0f - last_alpha) * acc1;
                    acc2 = last_alpha * lc2 + (1.0f - last_alpha) * acc2;
                    lc0 = col.x; lc1 = col.y; lc2 = col.z;
                    last_alpha = alpha;
                    float dL_dalpha = ((col.x - acc0) * gp0 + (col.y - acc1) * gp1 + (col.z - acc2) * gp2) * T -
                                      fT / one_m * dL_dfinal;
                    float wT = alpha * T;
                    v[0] = wT * gp0;
                    v[1] = wT * gp1;
                    v[2] = wT * gp2;
                    // A clamped alpha no longer depends on the gaussian (backward.cu:126-135).
                    if (pa.raw <= MAX_ALPHA) {
                        float dG = col.w * dL_dalpha * pa.G;
                        v[3] = pa.G * dL_dalpha;
                        v[4] = dG * (q.x * pa.dx + q.y * pa.dy);
                        v[5] = dG * (q.y * pa.dx + q.z * pa.dy);
                        v[6] = dG * (-0.5f * pa.dx * pa.dx);
                        v[7] = dG * (-pa.dx * pa.dy);
                        v8 = dG * (-0.5f * pa.dy * pa.dy);
                    }
                }
            }
            if (__any_sync(FULL_MASK, contributes)) {
                float total = warp_reduce_scatter8(v, lane);
                float t8 = warp_sum(v8);
                int g = s_id[k];
                if ((lane & 3) == 0 && total != 0.0f) {
                    int idx = lane >> 2;
                    float* dst = idx < 3 ? grad_colors + 3 * g + idx
                               : idx == 3 ? grad_opacities + g
                               : idx < 6 ? grad_means2D + 2 * g + (idx - 4)
                                         : grad_conics + 3 * g + (idx - 6);
                    atomicAdd(dst, total);
                }
                if (lane == 1 && t8 != 0.0f) atomicAdd(grad_conics + 3 * g + 2, t8);
            }
        }
    }
}

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" int hds_render_forward(int width, int height, int origin_y, const int32_t* tile_ranges,
                                  const int32_t* values_sorted,
                                  const float* means2D, const float* conic4, const float* color_opacity,
                                  const float* background, float* image4, float* final_T, int32_t* n_contrib,
                                  hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(width > 0 && height > 0, HDS_ERR_INVALID, "render_forward: bad image size %dx%d", width, height);
    HDS_REQUIRE(origin_y >= 0 && origin_y % TILE == 0, HDS_ERR_INVALID,
                "render_forward: origin_y %d must be a non-negative multiple of 16", origin_y);
    HDS_REQUIRE(((uintptr_t)image4 & 15) == 0 && ((uintptr_t)conic4 & 15) == 0 && ((uintptr_t)color_opacity & 15) == 0,
                HDS_ERR_INVALID, "render_forward: image4, conic4 and color_opacity must be 16-byte aligned");
    int tx = tiles_for(width), ty = tiles_for(height);
    rgb_forward_kernel<<<tx * ty, TILE_PIXELS, 0, stream>>>(
        width, height, tx, origin_y, reinterpret_cast<const int2*>(tile_ranges), values_sorted,
        reinterpret_cast<const float2*>(means2D), reinterpret_cast<const float4*>(conic4),
        reinterpret_cast<const float4*>(color_opacity), background, reinterpret_cast<float4*>(image4), final_T,
        n_contrib);
    HDS_CHECK_LAUNCH("rgb_forward_kernel");
    return HDS_OK;
}

extern "C" int hds_render_backward(int n, int width, int height, int origin_y, const float* grad_image,
                                   const float* means2D,
                                   const float* conic4, const float* color_opacity, const int32_t* values_sorted,
                                   const int32_t* tile_ranges, const float* final_T, const int32_t* n_contrib,
                                   const float* background, float* grad_means2D, float* grad_conics, float* grad_colors,
                                   float* grad_opacities, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0, HDS_ERR_INVALID, "render_backward: bad sizes");
    HDS_REQUIRE(origin_y >= 0 && origin_y % TILE == 0, HDS_ERR_INVALID,
                "render_backward: origin_y %d must be a non-negative multiple of 16", origin_y);
    if (n == 0) return HDS_OK;
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_means2D, 0, sizeof(float) * 2 * (size_t)n, stream));
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_conics, 0, sizeof(float) * 3 * (size_t)n, stream));
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_colors, 0, sizeof(float) * 3 * (size_t)n, stream));
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_opacities, 0, sizeof(float) * (size_t)n, stream));
    int tx = tiles_for(width), ty = tiles_for(height);
    rgb_backward_kernel<<<tx * ty, TILE_PIXELS, 0, stream>>>(
        width, height, tx, origin_y, reinterpret_cast<const int2*>(tile_ranges), values_sorted,
        reinterpret_cast<const float2*>(means2D), reinterpret_cast<const float4*>(conic4),
        reinterpret_cast<const float4*>(color_opacity), background, final_T, n_contrib, grad_image, grad_means2D,
        grad_conics, grad_colors, grad_opacities);
    HDS_CHECK_LAUNCH("rgb_backward_kernel");
    return HDS_OK;
}
