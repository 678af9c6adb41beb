// render_features.cu -- C-channel feature blend on tcgen05 TF32 tensor cores.
//
// Restates features.cu:116-346 of the reference (render_features + its host wrapper): every pixel
// blends its tile's sorted list front to back with the same alpha / transmittance walk as the RGB
// pass, and the feature image is out[p, c] = sum_j w[p, j] f[j, c] with w = alpha * T.
//
// Blackwell design.  A block owns half a 16x16 tile: 128 pixels, one per thread and one per TMEM
// lane.  The tile's list is consumed in chunks of 32 gaussians; a chunk holds only entries whose
// opacity-aware box touches the half tile (warp 0 compacts them, keeping each list position for
// the contributor count), and each warp skips the entries whose box misses its 8 x 4 pixels.
// Per chunk:
//   * every thread starts cp.async gathers of its share of the chunk's feature rows into the B
//     operand buffer, transposed to the K-major core-matrix layout (no registers held while they fly),
//   * walks the 32 gaussians for its pixel (FP32, the oracle's exact arithmetic), and writes the
//     TF32-rounded weights as four float4s of the A operand (K-major, conflict-free),
//   * rounds the landed feature rows to TF32 in place (cvt.rna; the tensor core would otherwise
//     truncate them),
//   * after a barrier, one thread issues 4 x (C / 256) tcgen05.mma (M = 128, N <= 256, K = 8) that
//     accumulate into TMEM, and commits them to the stage's mbarrier.
// Two stages alternate, so the tensor cores run chunk c while the threads prepare chunk c + 1.  The
// accumulators never leave TMEM until the epilogue reads them back with tcgen05.ld and stores the
// pixel's C channels.  The same walk optionally writes the RGB image, which the reference computes
// in a separate pass.
//
// Every mbarrier wait is bounded; a wait that runs out records HDS_ERR_DEVICE in g_status (read by
// hds_device_status), frees the block's TMEM and returns.
#include "hds_common.cuh"
#include "tcgen05.cuh"

namespace hds {

__device__ int g_status = 0;

namespace {

constexpr uint32_t WAIT_LIMIT = 1u << 22;

template <int C>
struct FwdCfg {
    static constexpr int PIX = 128;
    static constexpr int THREADS = 128;
    static constexpr int KC = 32;
    static constexpr int N_MMA = C < 256 ? C : 256;
    static constexpr int N_BLOCKS = C / N_MMA;
    static constexpr int TMEM_COLS = C;
    static constexpr int A_BYTES = PIX * KC * 4;
    static constexpr int B_BYTES = KC * C * 4;
    static constexpr int A_LBO = (PIX / 8) * 128;  // between K-quads: all 16 row groups of 8 rows x 16 B
    static constexpr int B_LBO = (C / 8) * 128;    // between K-quads: all C/8 groups of 8 channel rows x 16 B
    static constexpr int SMEM = 2 * (A_BYTES + B_BYTES) + 1024;
    // Both operands K-major: tf32 in MN-major layout is only readable with the 128B/32B-atom swizzle.
    static constexpr uint32_t IDESC = tc::idesc_tf32(128, N_MMA, false, false);
    static_assert(C == 32 || C == 64 || C == 128 || C == 256 || C == 512, "unsupported channel count");
};

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Lane of the (n+1)-th set bit of mask (n >= 0, fewer than popc(mask)).
__device__ __forceinline__ int nth_set_bit(unsigned mask, int n) {
    for (int i = 0; i < n; i++) mask &= mask - 1;
    return __ffs(mask) - 1;
}

template <int C>
__global__ void __launch_bounds__(128, 1) feature_forward_kernel(
    int width, int height, int tiles_x, const int2* __restrict__ ranges, const int32_t* __restrict__ values,
    const float2* __restrict__ means2D, const float4* __restrict__ conic4, const float4* __restrict__ color_opacity,
    const float* __restrict__ features, const float* __restrict__ background, float* __restrict__ feature_image,
    float* __restrict__ final_T, int32_t* __restrict__ n_contrib, float4* __restrict__ image4) {
    using Cfg = FwdCfg<C>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ int s_id[2][32];
    __shared__ float2 s_mean[2][32];
    __shared__ float4 s_conic[2][32];
    __shared__ float4 s_col[2][32];
    __shared__ float2 s_ext[2][32];
    __shared__ int s_pos[2][32];
    __shared__ int s_filled, s_cursor;
    __shared__ uint64_t s_bar[2];
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x >> 1;
    const int x0 = (tile % tiles_x) * TILE;
    const int y0 = (tile / tiles_x) * TILE + (blockIdx.x & 1) * 8;
    if (y0 >= height) return;  // the lower half of a bottom-row tile can lie wholly outside the image

    // Pixel of this thread (= A row = TMEM lane): warp w covers an 8 x 4 block of the 16 x 8 half tile.
    const int px = x0 + (warp & 1) * 8 + (lane & 7);
    const int py = y0 + (warp >> 1) * 4 + (lane >> 3);
    const bool inside = px < width && py < height;
    const float cx = (float)px + 0.5f, cy = (float)py + 0.5f;

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t a_base = tc::smem_addr(smem);
    const uint32_t b_base = a_base + 2 * Cfg::A_BYTES;

    if (warp == 0) tc::tmem_alloc(&s_tmem, Cfg::TMEM_COLS);
    if (tid == 0) {
        tc::mbar_init(&s_bar[0], 1);
        tc::mbar_init(&s_bar[1], 1);
        tc::fence_mbar_init();
        s_fail = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s_tmem;

    const int2 range = ranges[tile];
    const int count = range.y - range.x;
    const bool rgb = image4 != nullptr;
    // Pixel-centre rectangles of this block's half tile and of this warp's 8 x 4 pixel block.
    const float hx0 = (float)x0 + 0.5f, hx1 = hx0 + 15.0f, hy0 = (float)y0 + 0.5f, hy1 = hy0 + 7.0f;
    const float wx0 = (float)(x0 + (warp & 1) * 8) + 0.5f, wx1 = wx0 + 7.0f;
    const float wy0 = (float)(y0 + (warp >> 1) * 4) + 0.5f, wy1 = wy0 + 3.0f;

    float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f;
    int last = 0;
    bool done = !inside;
    int issued = 0;
    int cursor = 0;  // next list position to examine; every thread holds the same value

    for (int c = 0;; c++) {
        const int s = c & 1;
        // The stage's buffers are still read by the MMAs of chunk c - 2 until its commit arrives.
        if (tid == 0 && c >= 2 && !tc::mbar_wait_bounded(&s_bar[s], ((c - 2) >> 1) & 1, WAIT_LIMIT)) s_fail = 1;
        // Barrier: previous chunk fully consumed by this block's threads; stop when every pixel is done.
        if (__syncthreads_count(!done) == 0 || s_fail || cursor >= count) break;

        // Warp 0 fills the chunk with the next list entries whose opacity-aware box touches this
        // half tile (the others can never blend here), remembering each one's list position.
        if (warp == 0) {
            int filled = 0, cur = cursor;
            while (filled < Cfg::KC && cur < count) {
                const int pos = cur + lane;
                bool hit = false;
                int g = 0;
                float2 m = make_float2(0.0f, 0.0f), e = make_float2(0.0f, 0.0f);
                float4 q = make_float4(0.0f, 0.0f, 0.0f, 0.0f), col = q;
                if (pos < count) {
                    g = values[range.x + pos];
                    m = means2D[g];
                    q = conic4[g];
                    col = color_opacity[g];
                    e = cull_extent(q.x, q.y, q.z, col.w);
                    hit = box_hits(m, e, hx0, hx1, hy0, hy1);
                }
                const unsigned mask = __ballot_sync(FULL_MASK, hit);
                const int hits = __popc(mask);
                const int take = min(hits, Cfg::KC - filled);
                const int rank = __popc(mask & ((1u << lane) - 1u));
                if (hit && rank < take) {
                    const int slot = filled + rank;
                    s_id[s][slot] = g;
                    s_mean[s][slot] = m;
                    s_conic[s][slot] = q;
                    s_col[s][slot] = col;
                    s_ext[s][slot] = e;
                    s_pos[s][slot] = pos;
                }
                // When the chunk fills mid-batch, resume right after the last entry taken.
                cur = take < hits ? cur + nth_set_bit(mask, take - 1) + 1 : cur + 32;
                filled += take;
            }
            if (lane == 0) {
                s_filled = filled;
                s_cursor = min(cur, count);
            }
        }
        __syncthreads();
        const int valid = s_filled;
        cursor = s_cursor;
        if (valid == 0) break;  // nothing further in the list touches this half tile

        // B operand (K-major, no swizzle): element (k, n) at (k/4)*B_LBO + (n/8)*128 + (n%8)*16 + (k%4)*4,
        // so one 16-byte slot holds four consecutive gaussians of one channel.  Item i = (quad kq,
        // channel n = i % C): a warp fills 512 contiguous bytes, and each of its four 4-byte gathers
        // reads 128 contiguous bytes of one gaussian's feature row.  Unused rows are zeroed.
        const uint32_t b_stage = b_base + s * Cfg::B_BYTES;
        for (int i = tid; i < 8 * C; i += Cfg::THREADS) {
            const int n = i % C, kq = i / C;
            const uint32_t dst = b_stage + kq * Cfg::B_LBO + (n >> 3) * 128 + (n & 7) * 16;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int k = kq * 4 + e;
                if (k < valid)
                    cp_async4(dst + 4 * e, features + (size_t)s_id[s][k] * C + n);
                else
                    asm volatile("st.shared.f32 [%0], %1;" ::"r"(dst + 4 * e), "f"(0.0f) : "memory");
            }
        }
        cp_async_commit();

        // A operand (K-major, no swizzle): row m = tid, K-quad qd at qd*A_LBO + (m/8)*128 + (m%8)*16.
        // A warp whose 8 x 4 pixel block the gaussian's box misses skips it (weight 0 for all lanes).
        float* a_row = reinterpret_cast<float*>(smem + s * Cfg::A_BYTES + (tid >> 3) * 128 + (tid & 7) * 16);
#pragma unroll 1
        for (int qd = 0; qd < Cfg::KC / 4; qd++) {
            float w4[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int k = qd * 4 + e;
                float w = 0.0f;
                if (k < valid && !done && box_hits(s_mean[s][k], s_ext[s][k], wx0, wx1, wy0, wy1)) {
                    const float2 m = s_mean[s][k];
                    const float4 q = s_conic[s][k];
                    const float4 col = s_col[s][k];
                    PairAlpha pa = pair_alpha(cx, cy, m.x, m.y, q.x, q.y, q.z, col.w);
                    float alpha = fminf(MAX_ALPHA, pa.raw);
                    if (!(alpha < MIN_ALPHA)) {
                        float test = T * (1.0f - alpha);
                        if (test < MIN_T) {
                            done = true;
                        } else {
                            w = alpha * T;
                            if (rgb) {
                                ar = fmaf(w, col.x, ar);
                                ag = fmaf(w, col.y, ag);
                                ab = fmaf(w, col.z, ab);
                            }
                            T = test;
                            last = s_pos[s][k] + 1;
                        }
                    }
                }
                w4[e] = tc::to_tf32(w);
            }
            *reinterpret_cast<float4*>(a_row + qd * (Cfg::A_LBO / 4)) = make_float4(w4[0], w4[1], w4[2], w4[3]);
        }

        // Round this thread's landed feature slots to TF32 in place.
        cp_async_wait_all();
        for (int i = tid; i < 8 * C; i += Cfg::THREADS) {
            const int n = i % C, kq = i / C;
            float4* p = reinterpret_cast<float4*>(smem + 2 * Cfg::A_BYTES + s * Cfg::B_BYTES + kq * Cfg::B_LBO +
                                                  (n >> 3) * 128 + (n & 7) * 16);
            float4 v = *p;
            *p = make_float4(tc::to_tf32(v.x), tc::to_tf32(v.y), tc::to_tf32(v.z), tc::to_tf32(v.w));
        }
        tc::fence_proxy_async();
        __syncthreads();

        if (tid == 0) {
            tc::fence_after_sync();
            const uint32_t a_stage = a_base + s * Cfg::A_BYTES;
#pragma unroll
            for (int ks = 0; ks < Cfg::KC / 8; ks++) {
#pragma unroll
                for (int nb = 0; nb < Cfg::N_BLOCKS; nb++) {
                    uint64_t ad = tc::smem_desc(a_stage + ks * 2 * Cfg::A_LBO, Cfg::A_LBO, 128);
                    uint64_t bd =
                        tc::smem_desc(b_stage + ks * 2 * Cfg::B_LBO + nb * (Cfg::N_MMA / 8) * 128, Cfg::B_LBO, 128);
                    tc::mma_tf32(tmem + nb * Cfg::N_MMA, ad, bd, Cfg::IDESC, (c > 0 || ks > 0) ? 1u : 0u);
                }
            }
            tc::commit(&s_bar[s]);
        }
        issued = c + 1;
    }

    // Every issued MMA has completed once the last chunk's commit arrives.
    if (issued > 0 && tid == 0 && !s_fail &&
        !tc::mbar_wait_bounded(&s_bar[(issued - 1) & 1], ((issued - 1) >> 1) & 1, WAIT_LIMIT))
        s_fail = 1;
    __syncthreads();
    tc::fence_after_sync();
    const bool have = issued > 0 && !s_fail;

    const size_t p = (size_t)py * width + px;
    float* dst = feature_image + p * C;
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int col = 0; col < C; col += 16) {
        float v[16];
        if (have) {
            tc::tmem_ld16(lane_addr + col, v);  // warp-collective: every lane executes it
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = 0.0f;
        }
        if (inside) {
#pragma unroll
            for (int i = 0; i < 16; i += 4)
                *reinterpret_cast<float4*>(dst + col + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
    }
    if (inside) {
        final_T[p] = T;
        n_contrib[p] = last;
        if (rgb)
            image4[p] = make_float4(fmaf(T, background[0], ar), fmaf(T, background[1], ag), fmaf(T, background[2], ab),
                                    0.0f);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, Cfg::TMEM_COLS);
    if (tid == 0 && s_fail) atomicExch(&g_status, HDS_ERR_DEVICE);
}

template <int C>
int launch_forward(int width, int height, const int32_t* tile_ranges, const int32_t* values, const float* means2D,
                   const float* conic4, const float* color_opacity, const float* features, const float* background,
                   float* feature_image, float* final_T, int32_t* n_contrib, float* image4, cudaStream_t stream) {
    using Cfg = FwdCfg<C>;
    auto kernel = feature_forward_kernel<C>;
    HDS_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    int tx = tiles_for(width), ty = tiles_for(height);
    kernel<<<2 * tx * ty, Cfg::THREADS, Cfg::SMEM, stream>>>(
        width, height, tx, reinterpret_cast<const int2*>(tile_ranges), values, reinterpret_cast<const float2*>(means2D),
        reinterpret_cast<const float4*>(conic4), reinterpret_cast<const float4*>(color_opacity), features, background,
        feature_image, final_T, n_contrib, reinterpret_cast<float4*>(image4));
    HDS_CHECK_LAUNCH("feature_forward_kernel");
    return HDS_OK;
}

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" int hds_render_features_forward(int n, int channels, int width, int height, const int32_t* tile_ranges,
                                           const int32_t* values_sorted, const float* means2D, const float* conic4,
                                           const float* color_opacity, const float* features, const float* background,
                                           float* feature_image, float* final_T, int32_t* n_contrib, float* image4,
                                           hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0, HDS_ERR_INVALID, "rasterize_features: bad sizes");
    HDS_REQUIRE((int64_t)channels * width * height <= INT32_MAX, HDS_ERR_TOO_LARGE,
                "a %dx%d image of %d channels overflows the feature kernels' int indices", width, height, channels);
    HDS_REQUIRE(((uintptr_t)features & 15) == 0 && ((uintptr_t)feature_image & 15) == 0, HDS_ERR_INVALID,
                "rasterize_features: features and feature_image must be 16-byte aligned");
    HDS_REQUIRE(image4 == nullptr || (background != nullptr && ((uintptr_t)image4 & 15) == 0), HDS_ERR_INVALID,
                "rasterize_features: the fused RGB output needs a background and 16-byte alignment");
    switch (channels) {
        case 32: return launch_forward<32>(width, height, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, background, feature_image, final_T, n_contrib, image4, stream);
        case 64: return launch_forward<64>(width, height, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, background, feature_image, final_T, n_contrib, image4, stream);
        case 128: return launch_forward<128>(width, height, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, background, feature_image, final_T, n_contrib, image4, stream);
        case 256: return launch_forward<256>(width, height, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, background, feature_image, final_T, n_contrib, image4, stream);
        case 512: return launch_forward<512>(width, height, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, background, feature_image, final_T, n_contrib, image4, stream);
        default:
            set_error("features must have 32, 64, 128, 256 or 512 channels, got %d", channels);
            return HDS_ERR_UNSUPPORTED;
    }
}

extern "C" int hds_device_status(int* status, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(status != nullptr, HDS_ERR_INVALID, "device_status: null output");
    int zero = 0;
    HDS_CHECK_CUDA(cudaMemcpyFromSymbolAsync(status, g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream));
    HDS_CHECK_CUDA(cudaMemcpyToSymbolAsync(g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream));
    HDS_CHECK_CUDA(cudaStreamSynchronize(stream));
    return HDS_OK;
}
