// densify.cu -- densification on the device: the per-view statistics and the restructure of the
// parameter and Adam buffers that clone / split / prune produce (the reference's
// utils/gaussian.py:143-296, where both are host-driven torch indexing).
//
// Statistics (add_densification_stats, gaussian.py:143-160): for every gaussian the view rendered
// (radius > 0), max_radii2D = max(max_radii2D, radius), grad_accum += |dL/dmeans2D * (W/2, H/2)|
// (the gradient in normalised device coordinates) and denom += 1 -- one elementwise pass.
//
// Restructure: the caller decides which rows survive, which are copied and which become split
// children (the classification is a few elementwise tests), and hands over, per row of the new
// population, the source row, whether it is a split child and whether its Adam state starts at zero.
// One kernel then writes the new flat parameter buffer and both moment buffers segment by segment:
// every byte of the old buffers is read at most once per output row and every output byte is
// written once, coalesced along the row.  A split child's mean gets its offset added and its
// log-scales are replaced by log(exp(log_scale) / child_scale_div) (gaussian.py:245-256).
#include <algorithm>

#include "hds_common.cuh"

namespace hds {
namespace {

__global__ void __launch_bounds__(256) densify_stats_kernel(int n, const float2* __restrict__ grad_means2D,
                                                            const float* __restrict__ radii, float half_w,
                                                            float half_h, float* __restrict__ max_radii2D,
                                                            float* __restrict__ grad_accum,
                                                            float* __restrict__ denom) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float r = radii[i];
    if (!(r > 0.0f)) return;
    max_radii2D[i] = fmaxf(max_radii2D[i], r);
    const float2 g = grad_means2D[i];
    const float gx = g.x * half_w, gy = g.y * half_h;
    grad_accum[i] += sqrtf(gx * gx + gy * gy);
    denom[i] += 1.0f;
}

struct Segments {
    int count;
    int64_t old_offset[HDS_DENSIFY_MAX_SEGMENTS], new_offset[HDS_DENSIFY_MAX_SEGMENTS];
    int width[HDS_DENSIFY_MAX_SEGMENTS];
};

// blockIdx.y = segment; threads sweep that segment's n_new x width floats of the new buffers.
__global__ void __launch_bounds__(256) densify_apply_kernel(
    int n_new, int n_old, Segments seg, int means_segment, int log_scales_segment, float child_scale_div,
    const int32_t* __restrict__ src_row, const uint8_t* __restrict__ flags, const float* __restrict__ child_offset,
    const float* __restrict__ old_params, const float* __restrict__ old_m, const float* __restrict__ old_v,
    float* __restrict__ new_params, float* __restrict__ new_m, float* __restrict__ new_v) {
    const int s = blockIdx.y;
    const int w = seg.width[s];
    const int64_t total = (int64_t)n_new * w;
    const float* op = old_params + seg.old_offset[s];
    const float* om = old_m + seg.old_offset[s];
    const float* ov = old_v + seg.old_offset[s];
    float* np_ = new_params + seg.new_offset[s];
    float* nm = new_m + seg.new_offset[s];
    float* nv = new_v + seg.new_offset[s];
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (int64_t)gridDim.x * blockDim.x) {
        const int j = (int)(idx / w), e = (int)(idx - (int64_t)j * w);
        const int src = src_row[j];
        const uint8_t f = flags[j];
        const int64_t o = (int64_t)src * w + e;
        float p = op[o];
        if (f & HDS_DENSIFY_SPLIT_CHILD) {
            if (s == means_segment) p = p + child_offset[3 * (int64_t)j + e];
            if (s == log_scales_segment) p = logf(expf(p) / child_scale_div);
        }
        np_[idx] = p;
        const bool fresh = (f & HDS_DENSIFY_FRESH_STATE) != 0;
        nm[idx] = fresh ? 0.0f : om[o];
        nv[idx] = fresh ? 0.0f : ov[o];
    }
    (void)n_old;
}

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" int hds_densify_stats(int n, const float* grad_means2D, const float* radii, int width, int height,
                                 float* max_radii2D, float* grad_accum, float* denom, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0, HDS_ERR_INVALID, "densify_stats: bad sizes");
    HDS_REQUIRE(((uintptr_t)grad_means2D & 7) == 0, HDS_ERR_INVALID, "densify_stats: grad_means2D must be 8-byte aligned");
    if (n == 0) return HDS_OK;
    densify_stats_kernel<<<(n + 255) / 256, 256, 0, stream>>>(n, reinterpret_cast<const float2*>(grad_means2D), radii,
                                                              0.5f * (float)width, 0.5f * (float)height, max_radii2D,
                                                              grad_accum, denom);
    HDS_CHECK_LAUNCH("densify_stats_kernel");
    return HDS_OK;
}

extern "C" int hds_densify_apply(int n_old, int n_new, int segments, const int* widths, int means_segment,
                                 int log_scales_segment, float child_scale_div, const int32_t* src_row,
                                 const uint8_t* flags, const float* child_offset, const float* old_params,
                                 const float* old_exp_avg, const float* old_exp_avg_sq, float* new_params,
                                 float* new_exp_avg, float* new_exp_avg_sq, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n_old >= 0 && n_new >= 0, HDS_ERR_INVALID, "densify_apply: negative sizes");
    HDS_REQUIRE(segments >= 1 && segments <= HDS_DENSIFY_MAX_SEGMENTS && widths != nullptr, HDS_ERR_INVALID,
                "densify_apply: %d segments (1 to %d supported)", segments, HDS_DENSIFY_MAX_SEGMENTS);
    HDS_REQUIRE(means_segment < segments && log_scales_segment < segments, HDS_ERR_INVALID,
                "densify_apply: segment index out of range");
    HDS_REQUIRE(means_segment < 0 || widths[means_segment] == 3, HDS_ERR_INVALID,
                "densify_apply: the means segment must be 3 floats wide");
    HDS_REQUIRE(child_scale_div > 0.0f, HDS_ERR_INVALID, "densify_apply: child_scale_div must be positive");
    Segments seg{};
    seg.count = segments;
    int64_t old_off = 0, new_off = 0;
    for (int s = 0; s < segments; s++) {
        HDS_REQUIRE(widths[s] >= 1, HDS_ERR_INVALID, "densify_apply: segment %d has width %d", s, widths[s]);
        seg.width[s] = widths[s];
        seg.old_offset[s] = old_off;
        seg.new_offset[s] = new_off;
        old_off += (int64_t)n_old * widths[s];
        new_off += (int64_t)n_new * widths[s];
    }
    if (n_new == 0) return HDS_OK;
    HDS_REQUIRE(n_old > 0, HDS_ERR_INVALID, "densify_apply: new rows need old rows to copy");
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    dim3 grid((unsigned)std::min<int64_t>(((int64_t)n_new * 8 + 255) / 256, (int64_t)sms * 4), (unsigned)segments);
    densify_apply_kernel<<<grid, 256, 0, stream>>>(n_new, n_old, seg, means_segment, log_scales_segment,
                                                   child_scale_div, src_row, flags, child_offset, old_params,
                                                   old_exp_avg, old_exp_avg_sq, new_params, new_exp_avg,
                                                   new_exp_avg_sq);
    HDS_CHECK_LAUNCH("densify_apply_kernel");
    return HDS_OK;
}
