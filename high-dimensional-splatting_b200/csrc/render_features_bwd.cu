// render_features_bwd.cu -- backward of the feature blend.
//
// Restates features.cu:350-616 of the reference (render_features_backward + host wrapper): each
// pixel walks its tile's list back to front from its last contributor, recovering T by division,
// and produces dL/dfeatures (w * dL/dout summed over pixels), and dL/dalpha = T (dot - behind_dot)
// with dot = f . dL/dout, which drives the opacity, mean and conic gradients.
//
// Layout (the reference's "lane owns a channel slice"): a block owns one 16x16 tile and a slice of
// W channels; warp w owns an 8x4 pixel block and lane l owns channels l, l+32, ... of the slice for
// all 32 pixels of its warp, so dL/dout for (pixel, channel) sits in that lane's registers.  The
// feature gradient of a gaussian then accumulates inside one lane with no shuffles; shuffles are
// used only to finish the per-pixel dot (a 32-value reduce-scatter) and the six geometric
// gradients.  Gaussians whose opacity-aware box misses a warp's pixel block are skipped by ballot.
#include "hds_common.cuh"

namespace hds {
namespace {

constexpr int BWD_THREADS = 256;
constexpr int BWD_BATCH = 128;

__device__ __forceinline__ int2 warp_pixel(int warp, int lane) {
    return make_int2((warp & 1) * 8 + (lane & 7), (warp >> 1) * 4 + (lane >> 3));
}

// Sums V values over the warp, scattered: afterwards lane l holds the total of value l * V / 32
// (for V = 32 that is value l).  V is a power of two <= 32.
template <int V>
__device__ __forceinline__ float reduce_scatter(float* v, int lane) {
    int n = V;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        if (n > 1) {
            const bool hi = lane & o;
#pragma unroll
            for (int i = 0; i < V / 2; i++) {
                if (i < n / 2) {
                    float send = hi ? v[i] : v[i + n / 2];
                    float keep = hi ? v[i + n / 2] : v[i];
                    v[i] = keep + __shfl_xor_sync(FULL_MASK, send, o);
                }
            }
            n >>= 1;
        } else {
            v[0] += __shfl_xor_sync(FULL_MASK, v[0], o);
        }
    }
    return v[0];
}

template <int W>
__global__ void __launch_bounds__(BWD_THREADS, 1) feature_backward_kernel(
    int D, int width, int height, int tiles_x, const int2* __restrict__ ranges, const int32_t* __restrict__ values,
    const float2* __restrict__ means2D, const float4* __restrict__ conic4, const float4* __restrict__ color_opacity,
    const float* __restrict__ features, const float* __restrict__ final_T_in, const int32_t* __restrict__ n_contrib,
    const float* __restrict__ grad_out, float* __restrict__ grad_means2D, float* __restrict__ grad_conics,
    float* __restrict__ grad_features, float* __restrict__ grad_opacities) {
    constexpr int CPL = W / 32;
    const int slices = D / W;
    extern __shared__ float4 s_feat4[];
    __shared__ int s_id[BWD_BATCH];
    __shared__ float2 s_mean[BWD_BATCH];
    __shared__ float4 s_conic[BWD_BATCH];  // a, b, c, opacity
    __shared__ float2 s_ext[BWD_BATCH];
    __shared__ float s_w[BWD_THREADS];
    __shared__ int s_max_last;
    const float* s_feat = reinterpret_cast<const float*>(s_feat4);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x / slices;
    const int c0 = (blockIdx.x % slices) * W;
    const int x0 = (tile % tiles_x) * TILE, y0 = (tile / tiles_x) * TILE;
    const int2 lp = warp_pixel(warp, lane);
    const int px = x0 + lp.x, py = y0 + lp.y;
    const bool inside = px < width && py < height;
    const float cx = (float)px + 0.5f, cy = (float)py + 0.5f;
    const int p = py * width + px;
    // The warp's pixel-centre rectangle: lane 0 is its top-left pixel, lane 31 its bottom-right.
    const float rx0 = (float)(x0 + (warp & 1) * 8) + 0.5f, rx1 = rx0 + 7.0f;
    const float ry0 = (float)(y0 + (warp >> 1) * 4) + 0.5f, ry1 = ry0 + 3.0f;

    float grad[CPL][32];
#pragma unroll
    for (int q = 0; q < 32; q++) {
        int2 qp = warp_pixel(warp, q);
        int x = x0 + qp.x, y = y0 + qp.y;
        bool in = x < width && y < height;
#pragma unroll
        for (int i = 0; i < CPL; i++)
            grad[i][q] = in ? grad_out[(size_t)D * (y * width + x) + c0 + lane + 32 * i] : 0.0f;
    }
    float T = inside ? final_T_in[p] : 0.0f;
    const int last = inside ? n_contrib[p] : 0;
    const int2 range = ranges[tile];
    if (tid == 0) s_max_last = 0;
    __syncthreads();
    atomicMax(&s_max_last, last);
    __syncthreads();
    const int todo = min(range.y - range.x, s_max_last);

    float behind = 0.0f;
    for (int end = todo; end > 0; end -= BWD_BATCH) {
        const int n = min(BWD_BATCH, end);
        const int start = end - n;
        __syncthreads();
        if (tid < n) {
            int g = values[range.x + start + tid];
            s_id[tid] = g;
            s_mean[tid] = means2D[g];
            float4 q = conic4[g];
            float o = color_opacity[g].w;
            s_conic[tid] = make_float4(q.x, q.y, q.z, o);
            s_ext[tid] = cull_extent(q.x, q.y, q.z, o);
        }
        __syncthreads();
        for (int i = tid; i < n * (W / 4); i += BWD_THREADS) {
            int slot = i / (W / 4);
            s_feat4[i] = reinterpret_cast<const float4*>(features + (size_t)s_id[slot] * D + c0)[i % (W / 4)];
        }
        __syncthreads();

        for (int group = ((n - 1) >> 5) << 5; group >= 0; group -= 32) {
            const int cand = group + lane;
            bool hit = false;
            if (cand < n) {
                float2 m = s_mean[cand];
                float2 e = s_ext[cand];
                hit = box_hits(m, e, rx0, rx1, ry0, ry1);
            }
            unsigned mask = __ballot_sync(FULL_MASK, hit);
            while (mask) {
                const int bit = 31 - __clz(mask);
                mask &= ~(1u << bit);
                const int slot = group + bit;
                const float4 q = s_conic[slot];
                bool contributes = inside && start + slot < last;
                PairAlpha pa{0.0f, 0.0f, 0.0f, 0.0f};
                float alpha = 0.0f;
                if (contributes) {
                    float2 m = s_mean[slot];
                    pa = pair_alpha(cx, cy, m.x, m.y, q.x, q.y, q.z, q.w);
                    alpha = fminf(MAX_ALPHA, pa.raw);
                    contributes = alpha >= MIN_ALPHA;
                }
                if (!__any_sync(FULL_MASK, contributes)) continue;

                float f[CPL];
#pragma unroll
                for (int i = 0; i < CPL; i++) f[i] = s_feat[slot * W + lane + 32 * i];
                float part[32];
#pragma unroll
                for (int qq = 0; qq < 32; qq++) {
                    float acc = 0.0f;
#pragma unroll
                    for (int i = 0; i < CPL; i++) acc = fmaf(f[i], grad[i][qq], acc);
                    part[qq] = acc;
                }
                const float dot = reduce_scatter<32>(part, lane);

                float weight = 0.0f, dL_dalpha = 0.0f;
                if (contributes) {
                    T = T / (1.0f - alpha);
                    weight = T * alpha;
                    dL_dalpha = T * (dot - behind);
                    behind = alpha * dot + (1.0f - alpha) * behind;
                }
                float v[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
                if (contributes && pa.raw <= MAX_ALPHA) {
                    const float dG = q.w * dL_dalpha * pa.G;
                    v[0] = pa.G * dL_dalpha;
                    v[1] = dG * (q.x * pa.dx + q.y * pa.dy);
                    v[2] = dG * (q.y * pa.dx + q.z * pa.dy);
                    v[3] = dG * (-0.5f * pa.dx * pa.dx);
                    v[4] = dG * (-pa.dx * pa.dy);
                    v[5] = dG * (-0.5f * pa.dy * pa.dy);
                }
                const float total = reduce_scatter<8>(v, lane);
                const int g = s_id[slot];
                if ((lane & 3) == 0) {
                    const int k = lane >> 2;
                    if (k < 6 && total != 0.0f) {
                        float* dst = k == 0 ? grad_opacities + g : k < 3 ? grad_means2D + 2 * g + (k - 1)
                                                                         : grad_conics + 3 * g + (k - 3);
                        atomicAdd(dst, total);
                    }
                }
                s_w[tid] = weight;
                __syncwarp();
                float df[CPL];
#pragma unroll
                for (int i = 0; i < CPL; i++) df[i] = 0.0f;
#pragma unroll
                for (int qq = 0; qq < 32; qq++) {
                    const float wq = s_w[warp * 32 + qq];
#pragma unroll
                    for (int i = 0; i < CPL; i++) df[i] = fmaf(wq, grad[i][qq], df[i]);
                }
                __syncwarp();
#pragma unroll
                for (int i = 0; i < CPL; i++)
                    if (df[i] != 0.0f) atomicAdd(grad_features + (size_t)g * D + c0 + lane + 32 * i, df[i]);
            }
        }
    }
}

template <int W>
int launch_backward(int n, int D, int width, int height, const int32_t* tile_ranges, const int32_t* values,
                    const float* means2D, const float* conic4, const float* color_opacity, const float* features,
                    const float* final_T, const int32_t* n_contrib, const float* grad_output, float* grad_features,
                    float* grad_means2D, float* grad_conics, float* grad_opacities, cudaStream_t stream) {
    (void)n;
    const int smem = BWD_BATCH * W * (int)sizeof(float);
    auto kernel = feature_backward_kernel<W>;
    HDS_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    int tx = tiles_for(width), ty = tiles_for(height);
    kernel<<<tx * ty * (D / W), BWD_THREADS, smem, stream>>>(
        D, width, height, tx, reinterpret_cast<const int2*>(tile_ranges), values, reinterpret_cast<const float2*>(means2D),
        reinterpret_cast<const float4*>(conic4), reinterpret_cast<const float4*>(color_opacity), features, final_T,
        n_contrib, grad_output, grad_means2D, grad_conics, grad_features, grad_opacities);
    HDS_CHECK_LAUNCH("feature_backward_kernel");
    return HDS_OK;
}

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" int hds_render_features_backward(int n, int channels, int slice_width, int width, int height,
                                            const float* grad_output, const float* features, const float* means2D,
                                            const float* conic4, const float* color_opacity,
                                            const int32_t* values_sorted, const int32_t* tile_ranges,
                                            const float* final_T, const int32_t* n_contrib, float* grad_features,
                                            float* grad_means2D, float* grad_conics, float* grad_opacities,
                                            hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0, HDS_ERR_INVALID, "rasterize_features_backward: bad sizes");
    HDS_REQUIRE((int64_t)channels * width * height <= INT32_MAX, HDS_ERR_TOO_LARGE,
                "a %dx%d image of %d channels overflows the feature kernels' int indices", width, height, channels);
    // The (channels, slice) pairs the reference dispatches (features.cu:601-612).
    const int D = channels, Wd = slice_width;
    const bool supported = (D == 32 && Wd == 32) || (D == 64 && (Wd == 64 || Wd == 32)) ||
                           (D == 128 && (Wd == 128 || Wd == 64 || Wd == 32)) || (D == 256 && (Wd == 128 || Wd == 64)) ||
                           (D == 512 && (Wd == 128 || Wd == 64));
    HDS_REQUIRE(supported, HDS_ERR_UNSUPPORTED, "no feature backward for %d channels in slices of %d", D, Wd);
    HDS_REQUIRE(((uintptr_t)features & 15) == 0, HDS_ERR_INVALID, "rasterize_features_backward: features must be 16-byte aligned");
    if (n == 0) return HDS_OK;
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_features, 0, sizeof(float) * (size_t)n * D, stream));
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_means2D, 0, sizeof(float) * 2 * (size_t)n, stream));
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_conics, 0, sizeof(float) * 3 * (size_t)n, stream));
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_opacities, 0, sizeof(float) * (size_t)n, stream));
    switch (Wd) {
        case 32: return launch_backward<32>(n, D, width, height, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, final_T, n_contrib, grad_output, grad_features, grad_means2D, grad_conics, grad_opacities, stream);
        case 64: return launch_backward<64>(n, D, width, height, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, final_T, n_contrib, grad_output, grad_features, grad_means2D, grad_conics, grad_opacities, stream);
        default: return launch_backward<128>(n, D, width, height, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, final_T, n_contrib, grad_output, grad_features, grad_means2D, grad_conics, grad_opacities, stream);
    }
}
