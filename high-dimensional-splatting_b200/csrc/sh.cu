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


// Whole-block transfers: a block of SH_BLOCK gaussians holds SH_BLOCK * 3 floats of sh_dc and
// SH_BLOCK * 45 of sh_rest, both whole float4s.  Every thread issues all its 16-byte loads before its
// first shared-memory store, so that each thread keeps up to 13 loads in flight.
constexpr int DC_F4 = SH_BLOCK * 3 / 4;
constexpr int REST_F4 = SH_BLOCK * 45 / 4;
constexpr int REST_F4_PER_THREAD = (REST_F4 + SH_BLOCK - 1) / SH_BLOCK;
static_assert(SH_BLOCK * 3 % 4 == 0 && DC_F4 <= SH_BLOCK, "sh_dc of a block must be whole float4s");

__device__ __forceinline__ bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// Elements e..e+3 of a block's [SH_BLOCK, len] slice go to shared-memory rows at column offset + j.
__device__ __forceinline__ void scatter4(float* s, int e, int len, int offset, float4 v) {
    const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const int g = (e + c) / len;
        s[g * SH_STRIDE + offset + (e + c - g * len)] = vv[c];
    }
}

__device__ __forceinline__ float4 gather4(const float* s, int e, int len, int offset) {
    float vv[4];
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const int g = (e + c) / len;
        vv[c] = s[g * SH_STRIDE + offset + (e + c - g * len)];
    }
    return make_float4(vv[0], vv[1], vv[2], vv[3]);
}

// Copies the SH values of gaussians first..first+count-1 into shared-memory rows: w[j][c] of
// gaussian i at s_w[i * SH_STRIDE + j * 3 + c].  sh_rest is skipped when the degree is 0.
__device__ __forceinline__ void stage_sh(float* s_w, const float* __restrict__ sh_dc,
                                         const float* __restrict__ sh_rest, int first, int count, bool rest) {
    const float* dc = sh_dc + (size_t)first * 3;
    const float* rs = sh_rest + (size_t)first * 45;
    const int t = threadIdx.x;
    if (count == SH_BLOCK && aligned16(dc) && aligned16(rs)) {
        float4 d = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float4 r[REST_F4_PER_THREAD];
        if (t < DC_F4) d = __ldg(reinterpret_cast<const float4*>(dc) + t);
        if (rest) {
#pragma unroll
            for (int u = 0; u < REST_F4_PER_THREAD; u++) {
                const int q = t + u * SH_BLOCK;
                if (q < REST_F4) r[u] = __ldg(reinterpret_cast<const float4*>(rs) + q);
            }
        }
        if (t < DC_F4) scatter4(s_w, 4 * t, 3, 0, d);
        if (rest) {
#pragma unroll
            for (int u = 0; u < REST_F4_PER_THREAD; u++) {
                const int q = t + u * SH_BLOCK;
                if (q < REST_F4) scatter4(s_w, 4 * q, 45, 3, r[u]);
            }
        }
        return;
    }
    for (int e = t; e < count * 3; e += SH_BLOCK) s_w[(e / 3) * SH_STRIDE + e % 3] = dc[e];
    if (rest)
        for (int e = t; e < count * 45; e += SH_BLOCK) s_w[(e / 45) * SH_STRIDE + 3 + e % 45] = rs[e];
}

// Viewing direction of gaussian i.  Without a camera centre, src holds the unit directions [n,3].
// With one, src holds the means [n,3] and the direction is torch.nn.functional.normalize(means -
// camera_center, dim=-1) = x / max(|x|, 1e-12) (the reference's utils/gaussian.py:110); s receives
// the divisor for the backward.
__device__ __forceinline__ float3 view_dir(const float* __restrict__ src, const float* __restrict__ cam, int i,
                                           float& s) {
    float x = src[3 * i], y = src[3 * i + 1], z = src[3 * i + 2];
    s = 1.0f;
    if (cam == nullptr) return make_float3(x, y, z);
    x = x - __ldg(cam);
    y = y - __ldg(cam + 1);
    z = z - __ldg(cam + 2);
    s = fmaxf(sqrtf(x * x + y * y + z * z), 1e-12f);
    return make_float3(x / s, y / s, z / s);
}

// dL/d(means - camera_center) from dL/ddir: (g - dir (dir . g)) / s above the clamp, g / s at it.
__device__ __forceinline__ float3 view_dir_backward(float3 dir, float s, float3 g) {
    if (!(s > 1e-12f)) return make_float3(g.x / s, g.y / s, g.z / s);
    const float dot = dir.x * g.x + dir.y * g.y + dir.z * g.z;
    return make_float3((g.x - dir.x * dot) / s, (g.y - dir.y * dot) / s, (g.z - dir.z * dot) / s);
}

// dirs: unit directions, or the means when cam (the camera centre [3]) is given.
__global__ void __launch_bounds__(SH_BLOCK) sh_forward_kernel(int n, int k, const float* __restrict__ sh_dc,
                                                              const float* __restrict__ sh_rest, const float* __restrict__ dirs,
                                                              const float* __restrict__ cam, const float* __restrict__ radii,
                                                              float* __restrict__ rgb) {
    __shared__ float s_w[SH_BLOCK * SH_STRIDE];
    const int first = blockIdx.x * SH_BLOCK;
    const int count = min(SH_BLOCK, n - first);
    stage_sh(s_w, sh_dc, sh_rest, first, count, k > 1);
    __syncthreads();
    int i = first + threadIdx.x;
    if (threadIdx.x >= count) return;
    float3 out = make_float3(0.0f, 0.0f, 0.0f);
    if (radii[i] > 0.0f) {
        float b[16];
        float len;
        const float3 d = view_dir(dirs, cam, i, len);
        basis(d.x, d.y, d.z, b);
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
                                           float3 dir, const float* __restrict__ radii, float* g) {
    float3 dd = make_float3(0.0f, 0.0f, 0.0f);
    if (!(radii[i] > 0.0f)) {
        for (int t = 0; t < 48; t++) g[t] = 0.0f;
        return dd;
    }
    float b[16], bx[16], by[16], bz[16];
    const float x = dir.x, y = dir.y, z = dir.z;
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

// One Adam step of one element (sh.cu:90-102 of the reference: torch's Adam).
__device__ __forceinline__ void adam_element(float& p, float& m, float& v, float grad, float step_size,
                                             float bc2_sqrt, const Adam& a) {
    float mt = m + a.one_minus_beta1 * (grad - m);
    float vt = a.beta2 * v + a.one_minus_beta2 * grad * grad;
    m = mt;
    v = vt;
    p -= step_size * mt / (sqrtf(vt) / bc2_sqrt + a.eps);
}

// Adam on a block's contiguous [count, len] slice of a parameter and its moments; the gradient of
// element e is in shared-memory row e / len at column offset + e % len.
__device__ __forceinline__ void adam_slice(float* __restrict__ p, float* __restrict__ m, float* __restrict__ v,
                                           const float* g, int offset, int len, int count, float step, float lr,
                                           const Adam& a) {
    const float step_size = lr / (1.0f - powf(a.beta1, step));
    const float bc2_sqrt = sqrtf(1.0f - powf(a.beta2, step));
    const int total = count * len;
    if (count == SH_BLOCK && aligned16(p) && aligned16(m) && aligned16(v)) {
        // Whole float4s, four per thread per round with every load issued first.
        constexpr int ROUND = 4;
        for (int q0 = threadIdx.x; q0 < total / 4; q0 += ROUND * SH_BLOCK) {
            float4 pp[ROUND], mm[ROUND], vv[ROUND];
#pragma unroll
            for (int u = 0; u < ROUND; u++) {
                const int q = q0 + u * SH_BLOCK;
                if (q < total / 4) {
                    pp[u] = reinterpret_cast<const float4*>(p)[q];
                    mm[u] = reinterpret_cast<const float4*>(m)[q];
                    vv[u] = reinterpret_cast<const float4*>(v)[q];
                }
            }
#pragma unroll
            for (int u = 0; u < ROUND; u++) {
                const int q = q0 + u * SH_BLOCK;
                if (q < total / 4) {
                    const float4 gg = gather4(g, 4 * q, len, offset);
                    adam_element(pp[u].x, mm[u].x, vv[u].x, gg.x, step_size, bc2_sqrt, a);
                    adam_element(pp[u].y, mm[u].y, vv[u].y, gg.y, step_size, bc2_sqrt, a);
                    adam_element(pp[u].z, mm[u].z, vv[u].z, gg.z, step_size, bc2_sqrt, a);
                    adam_element(pp[u].w, mm[u].w, vv[u].w, gg.w, step_size, bc2_sqrt, a);
                    reinterpret_cast<float4*>(p)[q] = pp[u];
                    reinterpret_cast<float4*>(m)[q] = mm[u];
                    reinterpret_cast<float4*>(v)[q] = vv[u];
                }
            }
        }
        return;
    }
    for (int e = threadIdx.x; e < total; e += SH_BLOCK)
        adam_element(p[e], m[e], v[e], g[(e / len) * SH_STRIDE + offset + e % len], step_size, bc2_sqrt, a);
}

// A block's [count, len] gradient slice out of shared memory: written, or added to what dst holds.
template <bool ACCUMULATE>
__device__ __forceinline__ void store_grads(float* __restrict__ dst, const float* g, int offset, int len, int count) {
    const int total = count * len;
    if (count == SH_BLOCK && aligned16(dst)) {
        constexpr int PER_THREAD = (SH_BLOCK * 45 / 4 + SH_BLOCK - 1) / SH_BLOCK;
        float4 old[PER_THREAD];
        if (ACCUMULATE) {
#pragma unroll
            for (int u = 0; u < PER_THREAD; u++) {
                const int q = threadIdx.x + u * SH_BLOCK;
                if (q < total / 4) old[u] = reinterpret_cast<const float4*>(dst)[q];
            }
        }
#pragma unroll
        for (int u = 0; u < PER_THREAD; u++) {
            const int q = threadIdx.x + u * SH_BLOCK;
            if (q < total / 4) {
                float4 val = gather4(g, 4 * q, len, offset);
                if (ACCUMULATE) val = make_float4(old[u].x + val.x, old[u].y + val.y, old[u].z + val.z, old[u].w + val.w);
                reinterpret_cast<float4*>(dst)[q] = val;
            }
        }
        return;
    }
    for (int e = threadIdx.x; e < total; e += SH_BLOCK) {
        const float val = g[(e / len) * SH_STRIDE + offset + e % len];
        dst[e] = ACCUMULATE ? dst[e] + val : val;
    }
}

enum class ShGrad { Write, Accumulate, Adam };

// dirs: unit directions, or the means when cam (the camera centre [3]) is given; grad_dirs then
// receives dL/dmeans, added to what it holds in the Accumulate mode (dL/ddirs is always written).
template <ShGrad MODE>
__global__ void __launch_bounds__(SH_BLOCK) sh_backward_kernel(int n, int k, const float* __restrict__ grad_rgb,
                                                               float* sh_dc, float* sh_rest, const float* __restrict__ dirs,
                                                               const float* __restrict__ cam,
                                                               const float* __restrict__ radii, float* __restrict__ grad_dc,
                                                               float* __restrict__ grad_rest, float* __restrict__ grad_dirs,
                                                               float* m_dc, float* v_dc, float* m_rest, float* v_rest,
                                                               const float* step_dc, const float* step_rest, Adam adam) {
    // Each row holds a gaussian's SH values, then (in place) their gradients.
    __shared__ float s_w[SH_BLOCK * SH_STRIDE];
    float* s_g = s_w;
    const int first = blockIdx.x * SH_BLOCK;
    const int count = min(SH_BLOCK, n - first);
    // sh_grads reads no sh_rest value at degree 0 and writes all 48 gradients of a row.
    stage_sh(s_w, sh_dc, sh_rest, first, count, k > 1);
    __syncthreads();
    if (threadIdx.x < count) {
        int i = first + threadIdx.x;
        float len;
        const float3 dir = view_dir(dirs, cam, i, len);
        float3 dd = sh_grads(i, k, s_w + threadIdx.x * SH_STRIDE, grad_rgb, dir, radii, s_g + threadIdx.x * SH_STRIDE);
        if (cam != nullptr) {
            dd = view_dir_backward(dir, len, dd);
            if (MODE == ShGrad::Accumulate) {
                dd.x = grad_dirs[3 * i] + dd.x;
                dd.y = grad_dirs[3 * i + 1] + dd.y;
                dd.z = grad_dirs[3 * i + 2] + dd.z;
            }
        }
        grad_dirs[3 * i] = dd.x;
        grad_dirs[3 * i + 1] = dd.y;
        grad_dirs[3 * i + 2] = dd.z;
    }
    __syncthreads();
    if (MODE == ShGrad::Adam) {
        adam_slice(sh_dc + (size_t)first * 3, m_dc + (size_t)first * 3, v_dc + (size_t)first * 3, s_g, 0, 3, count,
                   *step_dc, adam.lr_dc, adam);
        adam_slice(sh_rest + (size_t)first * 45, m_rest + (size_t)first * 45, v_rest + (size_t)first * 45, s_g, 3, 45,
                   count, *step_rest, adam.lr_rest, adam);
    } else {
        store_grads<MODE == ShGrad::Accumulate>(grad_dc + (size_t)first * 3, s_g, 0, 3, count);
        store_grads<MODE == ShGrad::Accumulate>(grad_rest + (size_t)first * 45, s_g, 3, 45, count);
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
                                                                              sh_rest, dirs, nullptr, radii, rgb);
    HDS_CHECK_LAUNCH("sh_forward_kernel");
    return HDS_OK;
}

extern "C" int hds_eval_sh_backward(int n, int degree, const float* grad_rgb, const float* sh_dc, const float* sh_rest,
                                    const float* dirs, const float* radii, float* grad_sh_dc, float* grad_sh_rest,
                                    float* grad_dirs, hds_stream_t stream) {
    clear_error();
    if (int rc = check_degree(n, degree)) return rc;
    if (n == 0) return HDS_OK;
    sh_backward_kernel<ShGrad::Write><<<(n + SH_BLOCK - 1) / SH_BLOCK, SH_BLOCK, 0, stream>>>(
        n, (degree + 1) * (degree + 1), grad_rgb, const_cast<float*>(sh_dc), const_cast<float*>(sh_rest), dirs, nullptr,
        radii, grad_sh_dc, grad_sh_rest, grad_dirs, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, Adam{});
    HDS_CHECK_LAUNCH("sh_backward_kernel");
    return HDS_OK;
}

extern "C" int hds_eval_sh_backward_accumulate(int n, int degree, const float* grad_rgb, const float* sh_dc,
                                               const float* sh_rest, const float* dirs, const float* radii,
                                               float* grad_sh_dc, float* grad_sh_rest, float* grad_dirs,
                                               hds_stream_t stream) {
    clear_error();
    if (int rc = check_degree(n, degree)) return rc;
    if (n == 0) return HDS_OK;
    sh_backward_kernel<ShGrad::Accumulate><<<(n + SH_BLOCK - 1) / SH_BLOCK, SH_BLOCK, 0, stream>>>(
        n, (degree + 1) * (degree + 1), grad_rgb, const_cast<float*>(sh_dc), const_cast<float*>(sh_rest), dirs, nullptr,
        radii, grad_sh_dc, grad_sh_rest, grad_dirs, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, Adam{});
    HDS_CHECK_LAUNCH("sh_backward_accumulate_kernel");
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
    sh_backward_kernel<ShGrad::Adam><<<(n + SH_BLOCK - 1) / SH_BLOCK, SH_BLOCK, 0, stream>>>(
        n, (degree + 1) * (degree + 1), grad_rgb, sh_dc, sh_rest, dirs, nullptr, radii, nullptr, nullptr, grad_dirs, m_dc,
        v_dc,
        m_rest, v_rest, step_dc, step_rest, a);
    HDS_CHECK_LAUNCH("sh_backward_adam_kernel");
    return HDS_OK;
}

extern "C" int hds_eval_sh_forward_view(int n, int degree, const float* sh_dc, const float* sh_rest, const float* means,
                                        const float* camera_center, const float* radii, float* rgb,
                                        hds_stream_t stream) {
    clear_error();
    if (int rc = check_degree(n, degree)) return rc;
    HDS_REQUIRE(camera_center != nullptr, HDS_ERR_INVALID, "eval_sh_forward_view: camera_center is required");
    if (n == 0) return HDS_OK;
    sh_forward_kernel<<<(n + SH_BLOCK - 1) / SH_BLOCK, SH_BLOCK, 0, stream>>>(n, (degree + 1) * (degree + 1), sh_dc,
                                                                              sh_rest, means, camera_center, radii, rgb);
    HDS_CHECK_LAUNCH("sh_forward_kernel");
    return HDS_OK;
}

extern "C" int hds_eval_sh_backward_view(int n, int degree, const float* grad_rgb, const float* sh_dc,
                                         const float* sh_rest, const float* means, const float* camera_center,
                                         const float* radii, float* grad_sh_dc, float* grad_sh_rest, float* grad_means,
                                         int accumulate, hds_stream_t stream) {
    clear_error();
    if (int rc = check_degree(n, degree)) return rc;
    HDS_REQUIRE(camera_center != nullptr, HDS_ERR_INVALID, "eval_sh_backward_view: camera_center is required");
    if (n == 0) return HDS_OK;
    const int blocks = (n + SH_BLOCK - 1) / SH_BLOCK, k = (degree + 1) * (degree + 1);
    float* dc = const_cast<float*>(sh_dc);
    float* rest = const_cast<float*>(sh_rest);
    if (accumulate)
        sh_backward_kernel<ShGrad::Accumulate><<<blocks, SH_BLOCK, 0, stream>>>(
            n, k, grad_rgb, dc, rest, means, camera_center, radii, grad_sh_dc, grad_sh_rest, grad_means, nullptr,
            nullptr, nullptr, nullptr, nullptr, nullptr, Adam{});
    else
        sh_backward_kernel<ShGrad::Write><<<blocks, SH_BLOCK, 0, stream>>>(
            n, k, grad_rgb, dc, rest, means, camera_center, radii, grad_sh_dc, grad_sh_rest, grad_means, nullptr,
            nullptr, nullptr, nullptr, nullptr, nullptr, Adam{});
    HDS_CHECK_LAUNCH("sh_backward_kernel");
    return HDS_OK;
}
