/*
 * hds_b200.h -- C ABI of the B200 (sm_100a) high-dimensional gaussian splatting rasterizer.
 *
 * The library (libhds_b200.so) implements the hot path of alexkato29/high-dimensional-splatting:
 * EWA projection, SH colour, tile binning with a device radix sort, the RGB and C-channel
 * feature blends (feature contraction on tcgen05 TF32 tensor cores), their backward passes, and
 * fused SSIM.  Each entry point below replaces one entry point of the reference's torch extension
 * (gaussian_splatting/rasterizer/api.h, bound in bindings.cpp:4-43); the comment on each names the
 * reference function and its file:line.
 *
 * Conventions
 *  - Every pointer is a CUDA device pointer to contiguous row-major fp32 (or int32 / uint64 where
 *    typed) memory on the current device, laid out exactly as the reference's tensors.
 *  - Nothing here allocates device memory.  Where a step needs scratch, a *_scratch_bytes()
 *    query gives the size and the caller passes the buffer (256-byte aligned).
 *  - All work is queued on `stream` (a cudaStream_t; NULL is the legacy default stream) and is
 *    asynchronous, except hds_rasterize_prepare, which synchronises `stream` to read the number
 *    of (tile, gaussian) pairs -- the same host read as the reference (forward.cu:318-325).
 *  - Return value: HDS_OK (0) or an HDS_ERR_* code; hds_last_error() then describes the failure
 *    (thread-local; message texts match the reference's TORCH_CHECK wording where it has one).
 *  - Outputs are fully overwritten; gradient outputs are zero-filled by the call itself.
 */
#ifndef HDS_B200_H
#define HDS_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* hds_stream_t; /* cudaStream_t */

enum {
    HDS_OK = 0,
    HDS_ERR_INVALID = 1,     /* bad size, null pointer or misaligned buffer */
    HDS_ERR_UNSUPPORTED = 2, /* channel count / slice width outside the supported set */
    HDS_ERR_CUDA = 3,        /* a CUDA runtime call or kernel launch failed */
    HDS_ERR_SCRATCH = 4,     /* scratch buffer smaller than the *_scratch_bytes() query */
    HDS_ERR_TOO_LARGE = 5,   /* sizes beyond the int32 indexing of the reference's layouts */
    HDS_ERR_DEVICE = 6       /* a kernel recorded a device-side failure (bounded wait ran out) */
};

/* Thread-local description of the last failure on this thread ("" after success). */
const char* hds_last_error(void);

/* ABI version of this header (bumped on any signature change). */
int hds_abi_version(void);

/* Number of kernels this library has launched in the process so far (all threads and devices). */
unsigned long long hds_launch_count(void);
#define HDS_ABI_VERSION 3

/* ---------------------------------------------------------------------------------------------
 * Projection.  Replaces project_gaussians (projection.cu:210-231; autograd glue projection.py:25-96).
 * means/scales [n,3], quats [n,4] (w,x,y,z), opacities [n] (the [n,1] tensor), world_to_camera
 * [4,4] row-major on the device.  Outputs means2D [n,2], depths [n], radii [n] (0 = culled),
 * conics [n,3] (inverse 2-D covariance xx, xy, yy).
 * ------------------------------------------------------------------------------------------- */
int hds_project_forward(int n, const float* means, const float* scales, const float* quats, const float* opacities,
                        const float* world_to_camera, float fx, float fy, float cx, float cy, int width, int height,
                        float near_plane, float low_pass, float fov_scale, float* means2D, float* depths,
                        float* radii, float* conics, hds_stream_t stream);

/* Replaces project_gaussians_backward (projection.cu:234-253). */
int hds_project_backward(int n, const float* grad_means2D, const float* grad_conics, const float* means,
                         const float* scales, const float* quats, const float* world_to_camera, float fx, float fy,
                         float cx, float cy, int width, int height, float near_plane, float low_pass,
                         float fov_scale, float* grad_means, float* grad_scales, float* grad_quats,
                         hds_stream_t stream);

/* Projection of the model's raw parameters: log_scales [n,3], unnormalised quats [n,4] and opacity
 * logits [n] are activated in the kernel (scale = exp, quat = q / max(|q|, 1e-12), opacity =
 * sigmoid: the reference's utils/gaussian.py:73-98, which runs them as torch glue before
 * project_gaussians).  Also writes the activated opacities [n] that the blend takes. */
int hds_project_forward_raw(int n, const float* means, const float* log_scales, const float* quats,
                            const float* opacity_logits, const float* world_to_camera, float fx, float fy, float cx,
                            float cy, int width, int height, float near_plane, float low_pass, float fov_scale,
                            float* means2D, float* depths, float* radii, float* conics, float* opacities,
                            hds_stream_t stream);

/* Backward of hds_project_forward_raw: gradients of the raw parameters, through the activations.
 * grad_opacities (dL/d activated opacity, from the blend) may be NULL.  accumulate != 0 adds the four
 * gradients to what their buffers hold; 0 writes them. */
int hds_project_backward_raw(int n, const float* grad_means2D, const float* grad_conics, const float* grad_opacities,
                             const float* means, const float* log_scales, const float* quats,
                             const float* opacity_logits, const float* world_to_camera, float fx, float fy, float cx,
                             float cy, int width, int height, float near_plane, float low_pass, float fov_scale,
                             float* grad_means, float* grad_log_scales, float* grad_quats,
                             float* grad_opacity_logits, int accumulate, hds_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Spherical harmonics.  Replaces eval_sh (sh.cu:157-168; glue utils/sh.py:26-59).
 * sh_dc [n,1,3], sh_rest [n,15,3], dirs [n,3] unit vectors, radii [n]; rgb [n,3].
 * ------------------------------------------------------------------------------------------- */
int hds_eval_sh_forward(int n, int degree, const float* sh_dc, const float* sh_rest, const float* dirs,
                        const float* radii, float* rgb, hds_stream_t stream);

/* Replaces eval_sh_backward_adam (sh.cu:171-190; glue utils/sh.py:62-109): SH gradient kept on chip
 * and consumed by an in-place Adam step of sh_dc/sh_rest and their moments; returns dL/ddirs.
 * step_dc/step_rest are device scalars already incremented for this step (torch state["step"]).
 * one_minus_beta1/2 are 1 - beta formed in double by the caller, as torch does. */
int hds_eval_sh_backward_adam(int n, int degree, const float* grad_rgb, float* sh_dc, float* sh_rest,
                              const float* dirs, const float* radii, float* m_dc, float* v_dc, float* m_rest,
                              float* v_rest, const float* step_dc, const float* step_rest, float lr_dc, float lr_rest,
                              float beta1, float beta2, float one_minus_beta1, float one_minus_beta2, float eps,
                              float* grad_dirs, hds_stream_t stream);

/* Plain SH backward returning dL/dsh_dc [n,1,3], dL/dsh_rest [n,15,3] and dL/ddirs [n,3].  No
 * counterpart in the reference (which only has the fused-Adam form); data-parallel training needs
 * SH gradients it can all-reduce before any optimizer step. */
int hds_eval_sh_backward(int n, int degree, const float* grad_rgb, const float* sh_dc, const float* sh_rest,
                         const float* dirs, const float* radii, float* grad_sh_dc, float* grad_sh_rest,
                         float* grad_dirs, hds_stream_t stream);

/* hds_eval_sh_backward that adds dL/dsh_dc and dL/dsh_rest to what grad_sh_dc and grad_sh_rest hold
 * (dL/ddirs is written).  For loops that accumulate several views into one gradient buffer: it saves
 * a fresh [n,16,3] gradient and the separate add into the buffer.  No counterpart in the reference. */
int hds_eval_sh_backward_accumulate(int n, int degree, const float* grad_rgb, const float* sh_dc,
                                    const float* sh_rest, const float* dirs, const float* radii, float* grad_sh_dc,
                                    float* grad_sh_rest, float* grad_dirs, hds_stream_t stream);

/* SH colour with the viewing directions formed in the kernel: dirs = normalize(means - camera_center)
 * = x / max(|x|, 1e-12), the torch glue of the reference's Gaussian.colors (utils/gaussian.py:100-112)
 * fused into eval_sh.  means [n,3]; camera_center: 3 floats in device memory. */
int hds_eval_sh_forward_view(int n, int degree, const float* sh_dc, const float* sh_rest, const float* means,
                             const float* camera_center, const float* radii, float* rgb, hds_stream_t stream);

/* Backward of hds_eval_sh_forward_view: dL/dsh_dc, dL/dsh_rest and dL/dmeans (through the
 * normalisation).  accumulate != 0 adds all three to what the buffers hold; 0 writes them.  The
 * camera centre gets no gradient here (it is -sum dL/dmeans when the caller needs it). */
int hds_eval_sh_backward_view(int n, int degree, const float* grad_rgb, const float* sh_dc, const float* sh_rest,
                              const float* means, const float* camera_center, const float* radii, float* grad_sh_dc,
                              float* grad_sh_rest, float* grad_means, int accumulate, hds_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Binning + RGB blend.  Together these three calls replace rasterize (forward.cu:239-435).
 *
 * 1. hds_rasterize_prepare (forward.cu:284-326): culls, packs conic4 [n,4] = (a, b, c, 0) and
 *    color_opacity [n,4] = (r, g, b, opacity), counts the tiles each gaussian touches, sums the
 *    counts and writes the total number of (tile, gaussian) pairs to *num_duplicates (host).
 *    It synchronises `stream`.  scratch: hds_rasterize_prepare_scratch_bytes(n) bytes, which must
 *    stay untouched until hds_rasterize_sort has been queued.
 * 2. hds_rasterize_sort (forward.cu:340-404): writes values_sorted [num_duplicates] (gaussian ids)
 *    in the order of the reference's stable sort of the keys tile << 32 | depth bits -- every
 *    tile's list front to back, equal depths in gaussian order -- and tile_ranges [tiles,2]
 *    ([start, end), empty tiles 0, 0).  It reaches that order by a stable depth sort of the
 *    gaussians and a stable tile-id sort of the pairs emitted in depth order.  keys_sorted may be
 *    NULL; when given it receives the sorted 64-bit keys (bit-exactness checks).
 * 3. hds_render_forward (forward.cu:406-434): front-to-back FP32 blend.  image4 [H,W,4] (the
 *    reference's padded layout; channel 3 written 0), final_T [H,W], n_contrib [H,W] (1-based
 *    index of the last blended list entry).
 *
 * Bands of rows (origin_y; no counterpart in the reference).  Every call of the binning, blend and
 * backward entry points takes origin_y, the row of the full image at which this image's row 0 lies
 * (a non-negative multiple of 16; 0 renders a whole image, the reference's call).  With
 * origin_y = y0 and height = the band's rows, the call renders rows [y0, y0 + height) of the full
 * view: means2D stay in full-image pixels, pixel centres and tile rectangles use full-image
 * coordinates, and only the band's tile rows are binned, so the band's outputs equal those rows of
 * the full render bit for bit.  The tile-row split of one view across GPUs is built on it.
 * ------------------------------------------------------------------------------------------- */
size_t hds_rasterize_prepare_scratch_bytes(int n);
int hds_rasterize_prepare(int n, const float* means2D, const float* depths, const float* radii, const float* conics,
                          const float* colors, const float* opacities, int width, int height, int origin_y, float* conic4,
                          float* color_opacity, void* scratch, size_t scratch_bytes, int64_t* num_duplicates,
                          hds_stream_t stream);

size_t hds_rasterize_sort_scratch_bytes(int n, int64_t num_duplicates, int width, int height);
int hds_rasterize_sort(int n, int64_t num_duplicates, int width, int height, const void* prepare_scratch,
                       void* scratch, size_t scratch_bytes, int32_t* values_sorted, int32_t* tile_ranges,
                       uint64_t* keys_sorted, hds_stream_t stream);

int hds_render_forward(int width, int height, int origin_y, const int32_t* tile_ranges, const int32_t* values_sorted,
                       const float* means2D, const float* conic4, const float* color_opacity,
                       const float* background, float* image4, float* final_T, int32_t* n_contrib,
                       hds_stream_t stream);

/* Replaces rasterize_backward (backward.cu:166-226).  grad_image [H,W,3]; outputs dL/dmeans2D [n,2],
 * dL/dconics [n,3], dL/dcolors [n,3], dL/dopacities [n]. */
int hds_render_backward(int n, int width, int height, int origin_y, const float* grad_image, const float* means2D,
                        const float* conic4, const float* color_opacity, const int32_t* values_sorted,
                        const int32_t* tile_ranges, const float* final_T, const int32_t* n_contrib,
                        const float* background, float* grad_means2D, float* grad_conics, float* grad_colors,
                        float* grad_opacities, hds_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Feature blend.  Replaces rasterize_features (features.cu:299-346): features [n,C] with
 * C in {32, 64, 128, 256, 512} blended over a zero background into feature_image [H,W,C], plus its
 * own final_T and n_contrib.  The contraction runs on tcgen05 tensor cores in split bf16 (each weight
 * and feature as bf16 hi + lo, products hi*hi + hi*lo + lo*hi, fp32 accumulation).  When image4 is non-NULL the same walk also writes the RGB
 * image (colours from color_opacity, over `background`), which the reference computes in a second
 * pass; that is an addition, NULL reproduces the reference call.
 * ------------------------------------------------------------------------------------------- */
int hds_render_features_forward(int n, int channels, int width, int height, int origin_y, const int32_t* tile_ranges,
                                const int32_t* values_sorted, const float* means2D, const float* conic4,
                                const float* color_opacity, const float* features, const float* background,
                                float* feature_image, float* final_T, int32_t* n_contrib, float* image4,
                                hds_stream_t stream);

/* Replaces rasterize_features_backward (features.cu:561-616).  slice_width is the channel slice one
 * block owns, one of the reference's pairs (features.cu:601-612); any other pair is rejected.
 * Outputs dL/dfeatures [n,C], dL/dmeans2D [n,2], dL/dconics [n,3], dL/dopacities [n]. */
int hds_render_features_backward(int n, int channels, int slice_width, int width, int height, int origin_y,
                                 const float* grad_output, const float* features, const float* means2D,
                                 const float* conic4, const float* color_opacity, const int32_t* values_sorted,
                                 const int32_t* tile_ranges, const float* final_T, const int32_t* n_contrib,
                                 float* grad_features, float* grad_means2D, float* grad_conics,
                                 float* grad_opacities, hds_stream_t stream);

/* As hds_render_features_backward, but dL/dfeatures is ADDED to grad_features (which is not
 * cleared); the other three outputs are written as above.  No counterpart in the reference: it lets
 * a training loop that accumulates several views into one gradient buffer skip clearing a fresh
 * [n,C] buffer and adding it afterwards.  grad_features must be 16-byte aligned. */
int hds_render_features_backward_accumulate(int n, int channels, int slice_width, int width, int height,
                                            int origin_y, const float* grad_output, const float* features, const float* means2D,
                                            const float* conic4, const float* color_opacity,
                                            const int32_t* values_sorted, const int32_t* tile_ranges,
                                            const float* final_T, const int32_t* n_contrib, float* grad_features,
                                            float* grad_means2D, float* grad_conics, float* grad_opacities,
                                            hds_stream_t stream);

/* The RGB backward and the feature backward in one walk of the lists; no counterpart in the
 * reference, which runs rasterize_backward (backward.cu:7-164) and rasterize_features_backward
 * (features.cu:350-616) as two passes over the same lists.  Valid when the forward was the fused
 * one (hds_render_features_forward with image4), so both share final_T and n_contrib.
 *  - grad_image [H,W,3] with background [3]: the RGB terms; NULL leaves them out (then grad_colors
 *    is not touched and may be NULL).
 *  - grad_feature_image [H,W,C]: the feature terms; channels as hds_render_features_backward.
 *  - Outputs dL/dcolors [n,3], dL/dfeatures [n,C] (added to the buffer when accumulate_features is
 *    non-zero, otherwise overwritten), dL/dmeans2D [n,2], dL/dconics [n,3], dL/dopacities [n]: the
 *    sums of both passes.
 *  - workspace (256-byte aligned, workspace_bytes >= hds_backward_workspace_bytes(pairs, width,
 *    height), pairs = the frame's (tile, gaussian) pair count), or NULL: at 256 and 512 channels a
 *    first kernel cuts every half tile's list of contributing entries into it, which the walk then
 *    streams; without it every block cuts its own list from values_sorted.  The results are the same.
 *    A workspace too small for the frame's pairs leaves the lists empty and records HDS_ERR_TOO_LARGE
 *    in the device status (hds_device_status). */
int hds_render_backward_fused(int n, int channels, int width, int height, int origin_y, const float* grad_image,
                              const float* background, const float* grad_feature_image, const float* features,
                              const float* means2D, const float* conic4, const float* color_opacity,
                              const int32_t* values_sorted, const int32_t* tile_ranges, const float* final_T,
                              const int32_t* n_contrib, float* grad_colors, float* grad_features,
                              float* grad_means2D, float* grad_conics, float* grad_opacities,
                              int accumulate_features, void* workspace, size_t workspace_bytes, hds_stream_t stream);

/* Bytes of the hds_render_backward_fused workspace for a frame of `pairs` (tile, gaussian) pairs:
 * 48 bytes per pair and half tile plus a count per half tile.  No counterpart in the reference. */
size_t hds_backward_workspace_bytes(int64_t pairs, int width, int height);

/* ---------------------------------------------------------------------------------------------
 * SSIM (11x11 gaussian window, sigma 1.5).  Replace ssim_forward (ssim.cu:306-338) and
 * ssim_backward (ssim.cu:340-367); glue utils/loss.py:57-90.  Images [H,W,3]; grad_mean is a
 * device scalar (dL/d mean SSIM).
 * ------------------------------------------------------------------------------------------- */
int hds_ssim_forward(int height, int width, const float* rendered, const float* gt, float* ssim_map, float* d_mu,
                     float* d_aa, float* d_ab, hds_stream_t stream);
int hds_ssim_backward(int height, int width, const float* grad_mean, const float* rendered, const float* gt,
                      const float* d_mu, const float* d_aa, const float* d_ab, float* grad_rendered,
                      hds_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Optimizer step.  Replaces optimizer.step() of the reference's training loop (main.py:194:
 * torch.optim.Adam(fused=True, eps=1e-15), one parameter group per tensor, built by
 * utils/gaussian.py:123-139) with ONE kernel over flat buffers: params, exp_avg, exp_avg_sq and grads
 * each hold every parameter tensor back to back ([n] fp32).  Segment s covers
 * [segment_ends[s-1], segment_ends[s]) and steps with learning rate segment_lrs[s] (both host arrays,
 * at most HDS_ADAM_MAX_SEGMENTS; the last end must be n).  step counts from 1.  The element update is
 * the reference's Adam form (sh.cu:90-102): m += (1 - b1) (g - m); v = b2 v + (1 - b2) g g;
 * p -= lr / (1 - b1^step) * m / (sqrt(v) / sqrt(1 - b2^step) + eps), with one_minus_beta1/2 given by
 * the caller.  params, exp_avg and exp_avg_sq are updated in place.  16-byte aligned buffers move as
 * float4s; others element by element.
 * ------------------------------------------------------------------------------------------- */
#define HDS_ADAM_MAX_SEGMENTS 16
int hds_adam_step(int64_t n, float* params, float* exp_avg, float* exp_avg_sq, const float* grads, int segments,
                  const int64_t* segment_ends, const float* segment_lrs, float step, float beta1, float beta2,
                  float one_minus_beta1, float one_minus_beta2, float eps, hds_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Densification on the device.  Replace the host-driven torch indexing of utils/gaussian.py:143-296.
 *
 * hds_densify_stats (add_densification_stats, gaussian.py:143-160): for each gaussian with radius > 0,
 * max_radii2D = max(max_radii2D, radius), grad_accum += |dL/dmeans2D * (W/2, H/2)|, denom += 1.
 * All [n] fp32 (grad_means2D [n,2], 8-byte aligned).
 *
 * hds_densify_apply (the parameter and Adam surgery of _clone / _split / _prune, gaussian.py:194-296):
 * the old and new flat buffers hold `segments` parameter tensors back to back, segment s being
 * [n_old, widths[s]] (resp. [n_new, widths[s]]).  New row j copies old row src_row[j] of every segment
 * of params, exp_avg and exp_avg_sq; flags[j] & HDS_DENSIFY_FRESH_STATE zeroes its moments (appended
 * rows); flags[j] & HDS_DENSIFY_SPLIT_CHILD adds child_offset[j] (3 floats) to the means segment and
 * sets the log-scales segment to log(exp(log_scale) / child_scale_div).  means_segment /
 * log_scales_segment may be -1 (none).  widths is a host array; the rest are device pointers.
 * ------------------------------------------------------------------------------------------- */
#define HDS_DENSIFY_MAX_SEGMENTS 16
#define HDS_DENSIFY_SPLIT_CHILD 1
#define HDS_DENSIFY_FRESH_STATE 2
int hds_densify_stats(int n, const float* grad_means2D, const float* radii, int width, int height, float* max_radii2D,
                      float* grad_accum, float* denom, hds_stream_t stream);
int hds_densify_apply(int n_old, int n_new, int segments, const int* widths, int means_segment, int log_scales_segment,
                      float child_scale_div, const int32_t* src_row, const uint8_t* flags, const float* child_offset,
                      const float* old_params, const float* old_exp_avg, const float* old_exp_avg_sq, float* new_params,
                      float* new_exp_avg, float* new_exp_avg_sq, hds_stream_t stream);

/* Reads and clears the device-side failure word that kernels with bounded waits set (0 = none).
 * Synchronises `stream`. */
int hds_device_status(int* status, hds_stream_t stream);

/* ---------------------------------------------------------------------------------------------
 * Binning without any allocation.  No counterpart in the reference.
 *
 * For callers that cannot allocate device memory where they bin a frame.  Examples: a renderer
 * inside an application whose GPU memory belongs to another allocator, a real-time loop that must
 * not call cudaMalloc (it can synchronise the device), or an FFI host that only hands over
 * finished buffers.  Runs hds_rasterize_prepare followed by hds_rasterize_sort with their scratch
 * in a fixed file-scope device array of HDS_NOALLOC_SCRATCH_BYTES, so the caller passes only
 * inputs and outputs.
 *  - Outputs: conic4 [n,4], color_opacity [n,4], values_sorted (room for values_capacity entries),
 *    tile_ranges [tiles,2] and *num_duplicates (host).
 *  - Limits: sizes whose scratch would exceed the array (roughly 500K gaussians with 2M pairs)
 *    and pair counts above values_capacity are rejected with HDS_ERR_TOO_LARGE before any sort.
 *  - Memory: the array is 64 MiB per GPU that has called this function, held until the process
 *    exits.
 *  - Set-up: the first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress) with that device current.  Make that first call before any stream
 *    capture.
 *  - Sharing: every call reuses the same array, so calls that overlap on the GPU (other streams,
 *    other host threads) race and must be serialised by the caller.
 *  - Like hds_rasterize_prepare, it synchronises `stream` to read the pair count.
 * ------------------------------------------------------------------------------------------- */
#define HDS_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)
int hds_rasterize_bin_noalloc(int n, const float* means2D, const float* depths, const float* radii,
                              const float* conics, const float* colors, const float* opacities, int width, int height,
                              float* conic4, float* color_opacity, int32_t* values_sorted, int64_t values_capacity,
                              int32_t* tile_ranges, int64_t* num_duplicates, hds_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* HDS_B200_H */
