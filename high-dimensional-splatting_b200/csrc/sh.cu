// sh.cu -- real spherical harmonics (degree <= 3) colour per gaussian, its backward, and the
// backward fused with an in-place Adam step.
//
// Restates sh.cu:9-154 of the reference.  rgb_c = max(0.5 + sum_j b_j(dir) w_jc, 0), zero for culled
// gaussians.  The backward recomputes the colour to find the clamp, keeps the 48 SH gradients of a
// block's gaussians in shared memory and writes them (or the Adam update they drive) as one
// contiguous, coalesced sweep over the block's slice of sh_dc / sh_rest.
#include "hds_common.cuh"

namespace hds {
namespace {

constexpr int SH_BLOCK = 128;
// One gaussian's 48 SH values per shared-memory row, plus one pad word: with an odd stride the threads
// of a warp, each reading its own row, hit 32 different banks (a stride of 48 puts them on two).
constexpr int SH_STRIDE = 49;

// Real SH normalisation constants of degrees 0-3 (the standard table of the 3DGS code base).
__constant__ float SHC[16] = {
    0.28209479177387814f, -0.4886025119029199f, 0.4886025119029199f, -0.4886025119029199f,
    1.0925484305920792f, -1.0925484305920792f, 0.31539156525252005f, -1.0925484305920792f,
    0.5462742152960396f, -0.5900435899266435f, 2.890611442640554f, -0.4570457994644658f,
    0.3731763325901154f, -0.4570457994644658f, 1.445305721320277f, -0.5900435899266435f,
};

__device__ __forceinline__ void basis(float x, float y, float z, float* b) {
    float xx = x * x, yy = y * y, zz = z * z, xy = x * y, yz = y * z, xz = x * z;
    b[0] = SHC[0];
    b[1] = SHC[1] * y; b[2] = SHC[2] * z; b[3] = SHC[3] * x;
    b[4] = SHC[4] * xy; b[5] = SHC[5] * yz; b[6] = SHC[6] * (2.0f * zz - xx - yy);
    b[7] = SHC[7] * xz; b[8] = SHC[8] * (xx - yy);
    b[9] = SHC[9] * y * (3.0f * xx - yy); b[10] = SHC[10] * xy * z;
    b[11] = SHC[11] * y * (4.0f * zz - xx - yy);
    b[12] = SHC[12] * z * (2.0f * zz - 3.0f * xx - 3.0f * yy);
    b[13] = SHC[13] * x * (4.0f * zz - xx - yy);
    b[14] = SHC[14] * z * (xx - yy); b[15] = SHC[15] * x * (xx - 3.0f * yy);
}

__device__ __forceinline__ void basis_grad(float x, float y, float z, float* bx, float* by, float* bz) {
    float xx = x * x, yy = y * y, zz = z * z;
#pragma unroll
    for (int j = 0; j < 16; j++) bx[j] = by[j] = bz[j] = 0.0f;
    by[1] = SHC[1]; bz[2] = SHC[2]; bx[3] = SHC[3];
    bx[4] = SHC[4] * y; by[4] = SHC[4] * x;
    by[5] = SHC[5] * z; bz[5] = SHC[5] * y;
    bx[6] = SHC[6] * (-2.0f * x); by[6] = SHC[6] * (-2.0f * y); bz[6] = SHC[6] * (4.0f * z);
    bx[7] = SHC[7] * z; bz[7] = SHC[7] * x;
    bx[8] = SHC[8] * (2.0f * x); by[8] = SHC[8] * (-2.0f * y);
    bx[9] = SHC[9] * (6.0f * x * y); by[9] = SHC[9] * (3.0f * xx - 3.0f * yy);
    bx[10] = SHC[10] * y * z; by[10] = SHC[10] * x * z; bz[10] = SHC[10] * x * y;
    bx[11] = SHC[11] * (-2.0f * x * y); by[11] = SHC[11] * (4.0f * zz - xx - 3.0f * yy); bz[11] = SHC[11] * (8.0f * y * z);
    bx[12] = SHC[12] * (-6.0f * x * z); by[12] = SHC[12] * (-6.0f * y * z);
    bz[12] = SHC[12] * (6.0f * zz - 3.0f * xx - 3.0f * yy);
    bx[13] = SHC[13] * (4.0f * zz - 3.0f * xx - yy); by[13] = SHC[13] * (-2.0f * x * y); bz[13] = SHC[13] * (8.0f * x * z);
    bx[14] = SHC[14] * (2.0f * x * z); by[14] = SHC[14] * (-2.0f * y * z); bz[14] = SHC[14] * (xx - yy);
    bx[15] = SHC[15] * (3.0f * xx - 3.0f * yy); by[15] = SHC[15] * (-6.0f * x * y);
}


__global__ void __launch_bounds__(SH_BLOCK) sh_forward_kernel(int n, int k, const float* __restrict__ sh_dc,
                                                              const float* __restrict__ sh_rest, const float* __restrict__ dirs,
                                                              const float* __restrict__ radii, float* __restrict__ rgb) {
    __shared__ float s_w[SH_BLOCK * SH_STRIDE];
    const int first = blockIdx.x * SH_BLOCK;
    const int count = min(SH_BLOCK, n - first);
    // Interleave dc and rest per gaussian in shared memory: w[j][c] at s_w[i*SH_STRIDE + j*3 + c].
    for (int t = threadIdx.x; t < count * 3; t += SH_BLOCK)
        s_w[(t / 3) * SH_STRIDE + t % 3] = sh_dc[(size_t)first * 3 + t];
    if (k > 1)
        for (int t = threadIdx.x; t < count * 45; t += SH_BLOCK)
            s_w[(t / 45) * SH_STRIDE + 3 + t % 45] = sh_rest[(size_t)first * 45 + t];
    __syncthreads();
    int i = first + threadIdx.x;
    if (threadIdx.x >= count) return;
    float3 out = make_float3(0.0f, 0.0f, 0.0f);
    if (radii[i] > 0.0f) {
        float b[16];
        basis(dirs[3 * i], dirs[3 * i + 1], dirs[3 * i + 2], b);
        const float* w = s_w + threadIdx.x * SH_STRIDE;
        float v[3];
#pragma unroll
        for (int c = 0; c < 3; c++) {
            float value = 0.5f;
            for (int j = 0; j < k; j++) value += b[j] * w[j * 3 + c];
            v[c] = fmaxf(value, 0.0f);
        }
        out = make_float3(v[0], v[1], v[2]);
    }
    rgb[3 * i] = out.x;
    rgb[3 * i + 1] = out.y;
    rgb[3 * i + 2] = out.z;
}

// Gradients of one gaussian into shared memory (g[j*3+c], j < 16) and dL/ddir into registers.  g may
// be w itself: every w[j*3+c] is read before g[j*3+c] is written.
__device__ __forceinline__ float3 sh_grads(int i, int k, const float* w, const float* __restrict__ grad_rgb,
                                           const float* __restrict__ dirs, const float* __restrict__ radii, float* g) {
    float3 dd = make_float3(0.0f, 0.0f, 0.0f);
    if (!(radii[i] > 0.0f)) {
        for (int t = 0; t < 48; t++) g[t] = 0.0f;
        return dd;
    }
    float b[16], bx[16], by[16], bz[16];
    float x = dirs[3 * i], y = dirs[3 * i + 1], z = dirs[3 * i + 2];
    basis(x, y, z, b);
    basis_grad(x, y, z, bx, by, bz);
    float gc[3];
#pragma unroll
    for (int c = 0; c < 3; c++) {
        float value = 0.5f;
        for (int j = 0; j < k; j++) value += b[j] * w[j * 3 + c];
        gc[c] = value > 0.0f ? grad_rgb[3 * i + c] : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < 16; j++) {
        float t = 0.0f;
#pragma unroll
        for (int c = 0; c < 3; c++) {
            const float wv = j < k ? w[j * 3 + c] : 0.0f;
            g[j * 3 + c] = j < k ? b[j] * gc[c] : 0.0f;
            t += wv * gc[c];
        }
        if (j < k) { dd.x += t * bx[j]; dd.y += t * by[j]; dd.z += t * bz[j]; }
    }
    return dd;
}

struct Adam {
    float lr_dc, lr_rest, beta1, beta2, one_minus_beta1, one_minus_beta2, eps;
};

// sh.cu:90-102 of the reference: torch's Adam update on one contiguous slice.
__device__ __forceinline__ void adam_slice(float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
                                           const float* g, int stride, int offset, int len, int count, float step,
                                           float lr, const Adam& a) {
    float step_size = lr / (1.0f - powf(a.beta1, step));
    float bc2_sqrt = sqrtf(1.0f - powf(a.beta2, step));
    for (int t = threadIdx.x; t < count * len; t += SH_BLOCK) {
        float grad = g[(t / len) * stride + offset + t % len];
        float mt = m[t] + a.one_minus_beta1 * (grad - m[t]);
        float vt = a.beta2 * v[t] + a.one_minus_beta2 * grad * grad;
        m[t] = mt;
        v[t] = vt;
        p[t] -= step_size * mt / (sqrtf(vt) / bc2_sqrt + a.eps);
    }
}

template <bool ADAM>
__global__ void __launch_bounds__(SH_BLOCK) sh_backward_kernel(int n, int k, const float* __restrict__ grad_rgb,
                                                               float* sh_dc, float* sh_rest, const float* __restrict__ dirs,
                                                               const float* __restrict__ radii, float* __restrict__ grad_dc,
                                                               float* __restrict__ grad_rest, float* __restrict__ grad_dirs,
                                                               float* m_dc, float* v_dc, float* m_rest, float* v_rest,
                                                               const float* step_dc, const float* step_rest, Adam adam) {
    // Each row holds a gaussian's SH values, then (in place) their gradients.
    __shared__ float s_w[SH_BLOCK * SH_STRIDE];
    float* s_g = s_w;
    const int first = blockIdx.x * SH_BLOCK;
    const int count = min(SH_BLOCK, n - first);
    for (int t = threadIdx.x; t < count * 3; t += SH_BLOCK)
        s_w[(t / 3) * SH_STRIDE + t % 3] = sh_dc[(size_t)first * 3 + t];
    for (int t = threadIdx.x; t < count * 45; t += SH_BLOCK)
        s_w[(t / 45) * SH_STRIDE + 3 + t % 45] = sh_rest[(size_t)first * 45 + t];
    __syncthreads();
    if (threadIdx.x < count) {
        int i = first + threadIdx.x;
        float3 dd = sh_grads(i, k, s_w + threadIdx.x * SH_STRIDE, grad_rgb, dirs, radii, s_g + threadIdx.x * SH_STRIDE);
        grad_dirs[3 * i] = dd.x;
        grad_dirs[3 * i + 1] = dd.y;
        grad_dirs[3 * i + 2] = dd.z;
    }
    __syncthreads();
    if (ADAM) {
        adam_slice(sh_dc + (size_t)first * 3, m_dc + (size_t)first * 3, v_dc + (size_t)first * 3, s_g, SH_STRIDE, 0, 3, count,
                   *step_dc, adam.lr_dc, adam);
        adam_slice(sh_rest + (size_t)first * 45, m_rest + (size_t)first * 45, v_rest + (size_t)first * 45, s_g, SH_STRIDE, 3, 45,
                   count, *step_rest, adam.lr_rest, adam);
    } else {
        for (int t = threadIdx.x; t < count * 3; t += SH_BLOCK)
            grad_dc[(size_t)first * 3 + t] = s_g[(t / 3) * SH_STRIDE + t % 3];
        for (int t = threadIdx.x; t < count * 45; t += SH_BLOCK)
            grad_rest[(size_t)first * 45 + t] = s_g[(t / 45) * SH_STRIDE + 3 + t % 45];
    }
}

int check_degree(int n, int degree) {
    HDS_REQUIRE(n >= 0, HDS_ERR_INVALID, "eval_sh: n must be >= 0, got %d", n);
    HDS_REQUIRE(degree >= 0 && degree <= 3, HDS_ERR_INVALID, "eval_sh: degree must be 0..3, got %d", degree);
    return HDS_OK;
}

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" int hds_eval_sh_forward(int n, int degree, const float* sh_dc, const float* sh_rest, const float* dirs,
                                   const float* radii, float* rgb, hds_stream_t stream) {
    clear_error();
    if (int rc = check_degree(n, degree)) return rc;
    if (n == 0) return HDS_OK;
    sh_forward_kernel<<<(n + SH_BLOCK - 1) / SH_BLOCK, SH_BLOCK, 0, stream>>>(n, (degree + 1) * (degree + 1), sh_dc,
                                                                              sh_rest, dirs, radii, rgb);
    HDS_CHECK_LAUNCH("sh_forward_kernel");
    return HDS_OK;
}

extern "C" int hds_eval_sh_backward(int n, int degree, const float* grad_rgb, const float* sh_dc, const float* sh_rest,
                                    const float* dirs, const float* radii, float* grad_sh_dc, float* grad_sh_rest,
                                    float* grad_dirs, hds_stream_t stream) {
    clear_error();
    if (int rc = check_degree(n, degree)) return rc;
    if (n == 0) return HDS_OK;
    sh_backward_kernel<false><<<(n + SH_BLOCK - 1) / SH_BLOCK, SH_BLOCK, 0, stream>>>(
        n, (degree + 1) * (degree + 1), grad_rgb, const_cast<float*>(sh_dc), const_cast<float*>(sh_rest), dirs, radii,
        grad_sh_dc, grad_sh_rest, grad_dirs, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, Adam{});
    HDS_CHECK_LAUNCH("sh_backward_kernel");
    return HDS_OK;
}

extern "C" int hds_eval_sh_backward_adam(int n, int degree, const float* grad_rgb, float* sh_dc, float* sh_rest,
                                         const float* dirs, const float* radii, float* m_dc, float* v_dc, float* m_rest,
                                         float* v_rest, const float* step_dc, const float* step_rest, float lr_dc,
                                         float lr_rest, float beta1, float beta2, float one_minus_beta1,
                                         float one_minus_beta2, float eps, float* grad_dirs, hds_stream_t stream) {
    clear_error();
    if (int rc = check_degree(n, degree)) return rc;
    if (n == 0) return HDS_OK;
    Adam a{lr_dc, lr_rest, beta1, beta2, one_minus_beta1, one_minus_beta2, eps};
    sh_backward_kernel<true><<<(n + SH_BLOCK - 1) / SH_BLOCK, SH_BLOCK, 0, stream>>>(
        n, (degree + 1) * (degree + 1), grad_rgb, sh_dc, sh_rest, dirs, radii, nullptr, nullptr, grad_dirs, m_dc, v_dc,
        m_rest, v_rest, step_dc, step_rest, a);
    HDS_CHECK_LAUNCH("sh_backward_adam_kernel");
    return HDS_OK;
}
