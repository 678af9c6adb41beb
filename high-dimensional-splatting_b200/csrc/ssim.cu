// ssim.cu -- fused SSIM (11-tap gaussian window, sigma 1.5) forward and backward.
//
// Restates ssim.cu:6-177 of the reference.  The reference runs two kernels per direction and keeps
// five (forward) or three (backward) blurred planes in HBM between them; here one block computes a
// 32 x 16 output tile: it stages the tile plus a 5-pixel halo in shared memory, blurs rows into
// shared memory, blurs columns, and writes only the results.  Out-of-image taps are zero-padded,
// which adds exact zeros where the reference skips the tap, so sums round identically.
#include "hds_common.cuh"

namespace hds {
namespace {

constexpr int R = 5;
constexpr int TX = 32, TY = 16;
constexpr int HX = TX + 2 * R, HY = TY + 2 * R;  // 42 x 26 staged pixels
constexpr int SSIM_THREADS = 256;
constexpr float C1 = 0.01f * 0.01f;
constexpr float C2 = 0.03f * 0.03f;

// Normalised exp(-x^2 / (2 * 1.5^2)), x = -5..5, rounded to float (the reference's ssim.cu:12-15).
__constant__ float GW[11];

__device__ __forceinline__ int sidx(int y, int x, int c) { return (y * HX + x) * 3 + c; }
__device__ __forceinline__ int hidx(int y, int x, int c) { return (y * TX + x) * 3 + c; }

__global__ void __launch_bounds__(SSIM_THREADS) ssim_forward_kernel(int height, int width, const float* __restrict__ a,
                                                                    const float* __restrict__ b, float* __restrict__ ssim_map,
                                                                    float* __restrict__ d_mu, float* __restrict__ d_aa,
                                                                    float* __restrict__ d_ab) {
    extern __shared__ float sm[];
    float* sa = sm;                   // [HY][HX][3]
    float* sb = sa + HY * HX * 3;     // [HY][HX][3]
    float* h = sb + HY * HX * 3;      // 5 planes [HY][TX][3]
    const int plane = HY * TX * 3;
    const int gx0 = blockIdx.x * TX - R, gy0 = blockIdx.y * TY - R;
    for (int i = threadIdx.x; i < HY * HX * 3; i += SSIM_THREADS) {
        int c = i % 3, x = (i / 3) % HX, y = i / (3 * HX);
        int gx = gx0 + x, gy = gy0 + y;
        bool in = gx >= 0 && gx < width && gy >= 0 && gy < height;
        size_t g = ((size_t)gy * width + gx) * 3 + c;
        sa[i] = in ? a[g] : 0.0f;
        sb[i] = in ? b[g] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < HY * TX * 3; i += SSIM_THREADS) {
        int c = i % 3, x = (i / 3) % TX, y = i / (3 * TX);
        float s_a = 0.0f, s_b = 0.0f, s_aa = 0.0f, s_bb = 0.0f, s_ab = 0.0f;
#pragma unroll
        for (int k = 0; k < 11; k++) {
            float va = sa[sidx(y, x + k, c)], vb = sb[sidx(y, x + k, c)];
            float wa = GW[k] * va, wb = GW[k] * vb;
            s_a += wa;
            s_b += wb;
            s_aa = fmaf(wa, va, s_aa);
            s_bb = fmaf(wb, vb, s_bb);
            s_ab = fmaf(wa, vb, s_ab);
        }
        h[i] = s_a; h[plane + i] = s_b; h[2 * plane + i] = s_aa; h[3 * plane + i] = s_bb; h[4 * plane + i] = s_ab;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < TY * TX * 3; i += SSIM_THREADS) {
        int c = i % 3, x = (i / 3) % TX, y = i / (3 * TX);
        int gx = blockIdx.x * TX + x, gy = blockIdx.y * TY + y;
        if (gx >= width || gy >= height) continue;
        float mu_a = 0.0f, mu_b = 0.0f, e_aa = 0.0f, e_bb = 0.0f, e_ab = 0.0f;
#pragma unroll
        for (int k = 0; k < 11; k++) {
            int j = hidx(y + k, x, c);
            float wk = GW[k];
            mu_a = fmaf(wk, h[j], mu_a);
            mu_b = fmaf(wk, h[plane + j], mu_b);
            e_aa = fmaf(wk, h[2 * plane + j], e_aa);
            e_bb = fmaf(wk, h[3 * plane + j], e_bb);
            e_ab = fmaf(wk, h[4 * plane + j], e_ab);
        }
        float mab = mu_a * mu_b, maa = mu_a * mu_a, mbb = mu_b * mu_b;
        float a1 = 2.0f * mab + C1;
        float a2 = 2.0f * (e_ab - mab) + C2;
        float b1 = maa + mbb + C1;
        float b2 = (e_aa - maa) + (e_bb - mbb) + C2;
        float inv_b = 1.0f / (b1 * b2);
        float s = a1 * a2 * inv_b;
        size_t g = ((size_t)gy * width + gx) * 3 + c;
        ssim_map[g] = s;
        d_mu[g] = (2.0f * mu_b * (a2 - a1) - 2.0f * mu_a * s * (b2 - b1)) * inv_b;
        d_aa[g] = -s / b2;
        d_ab[g] = 2.0f * a1 * inv_b;
    }
}

__global__ void __launch_bounds__(SSIM_THREADS) ssim_backward_kernel(int height, int width, const float* __restrict__ grad_mean,
                                                                     const float* __restrict__ a, const float* __restrict__ b,
                                                                     const float* __restrict__ d_mu, const float* __restrict__ d_aa,
                                                                     const float* __restrict__ d_ab, float* __restrict__ grad) {
    extern __shared__ float sm[];
    float* p_mu = sm;                  // [HY][HX][3] each
    float* p_aa = p_mu + HY * HX * 3;
    float* p_ab = p_aa + HY * HX * 3;
    float* h = p_ab + HY * HX * 3;     // 3 planes [HY][TX][3]
    const int plane = HY * TX * 3;
    const int gx0 = blockIdx.x * TX - R, gy0 = blockIdx.y * TY - R;
    for (int i = threadIdx.x; i < HY * HX * 3; i += SSIM_THREADS) {
        int c = i % 3, x = (i / 3) % HX, y = i / (3 * HX);
        int gx = gx0 + x, gy = gy0 + y;
        bool in = gx >= 0 && gx < width && gy >= 0 && gy < height;
        size_t g = ((size_t)gy * width + gx) * 3 + c;
        p_mu[i] = in ? d_mu[g] : 0.0f;
        p_aa[i] = in ? d_aa[g] : 0.0f;
        p_ab[i] = in ? d_ab[g] : 0.0f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < HY * TX * 3; i += SSIM_THREADS) {
        int c = i % 3, x = (i / 3) % TX, y = i / (3 * TX);
        float s_mu = 0.0f, s_aa = 0.0f, s_ab = 0.0f;
#pragma unroll
        for (int k = 0; k < 11; k++) {
            int j = sidx(y, x + k, c);
            float wk = GW[k];
            s_mu = fmaf(wk, p_mu[j], s_mu);
            s_aa = fmaf(wk, p_aa[j], s_aa);
            s_ab = fmaf(wk, p_ab[j], s_ab);
        }
        h[i] = s_mu; h[plane + i] = s_aa; h[2 * plane + i] = s_ab;
    }
    __syncthreads();
    const float scale = grad_mean[0] / (float)(height * width * 3);
    for (int i = threadIdx.x; i < TY * TX * 3; i += SSIM_THREADS) {
        int c = i % 3, x = (i / 3) % TX, y = i / (3 * TX);
        int gx = blockIdx.x * TX + x, gy = blockIdx.y * TY + y;
        if (gx >= width || gy >= height) continue;
        float s_mu = 0.0f, s_aa = 0.0f, s_ab = 0.0f;
#pragma unroll
        for (int k = 0; k < 11; k++) {
            int j = hidx(y + k, x, c);
            float wk = GW[k];
            s_mu = fmaf(wk, h[j], s_mu);
            s_aa = fmaf(wk, h[plane + j], s_aa);
            s_ab = fmaf(wk, h[2 * plane + j], s_ab);
        }
        size_t g = ((size_t)gy * width + gx) * 3 + c;
        grad[g] = scale * (s_mu + 2.0f * a[g] * s_aa + b[g] * s_ab);
    }
}

int upload_window(cudaStream_t stream) {
    // The window is formed in double on the host and rounded once, like the reference's constants.
    static float w[11];
    static bool ready = false;
    if (!ready) {
        double g[11], s = 0.0;
        for (int k = 0; k < 11; k++) {
            double x = k - 5;
            g[k] = exp(-x * x / (2.0 * 1.5 * 1.5));
            s += g[k];
        }
        for (int k = 0; k < 11; k++) w[k] = (float)(g[k] / s);
        ready = true;
    }
    HDS_CHECK_CUDA(cudaMemcpyToSymbolAsync(GW, w, sizeof(w), 0, cudaMemcpyHostToDevice, stream));
    return HDS_OK;
}

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" int hds_ssim_forward(int height, int width, const float* rendered, const float* gt, float* ssim_map,
                                float* d_mu, float* d_aa, float* d_ab, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(height > 0 && width > 0 && (int64_t)height * width * 3 <= INT32_MAX, HDS_ERR_INVALID,
                "ssim inputs must both be [H, W, 3] (got %dx%d)", height, width);
    if (int rc = upload_window(stream)) return rc;
    const int smem = (2 * HY * HX * 3 + 5 * HY * TX * 3) * (int)sizeof(float);
    HDS_CHECK_CUDA(cudaFuncSetAttribute(ssim_forward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    dim3 grid((width + TX - 1) / TX, (height + TY - 1) / TY);
    ssim_forward_kernel<<<grid, SSIM_THREADS, smem, stream>>>(height, width, rendered, gt, ssim_map, d_mu, d_aa, d_ab);
    HDS_CHECK_LAUNCH("ssim_forward_kernel");
    return HDS_OK;
}

extern "C" int hds_ssim_backward(int height, int width, const float* grad_mean, const float* rendered, const float* gt,
                                 const float* d_mu, const float* d_aa, const float* d_ab, float* grad_rendered,
                                 hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(height > 0 && width > 0 && (int64_t)height * width * 3 <= INT32_MAX, HDS_ERR_INVALID,
                "ssim inputs must both be [H, W, 3] (got %dx%d)", height, width);
    if (int rc = upload_window(stream)) return rc;
    const int smem = (3 * HY * HX * 3 + 3 * HY * TX * 3) * (int)sizeof(float);
    HDS_CHECK_CUDA(cudaFuncSetAttribute(ssim_backward_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    dim3 grid((width + TX - 1) / TX, (height + TY - 1) / TY);
    ssim_backward_kernel<<<grid, SSIM_THREADS, smem, stream>>>(height, width, grad_mean, rendered, gt, d_mu, d_aa, d_ab,
                                                               grad_rendered);
    HDS_CHECK_LAUNCH("ssim_backward_kernel");
    return HDS_OK;
}
