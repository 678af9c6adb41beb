// projection.cu -- EWA projection of 3-D gaussians into the image plane and its analytic backward.
//
// Restates projection.cu:13-197 of the reference: world->camera transform, perspective Jacobian
// with the ratio clamped to fov_scale * half the field of view, 2-D covariance T T^T plus a
// low-pass term, conic = inverse covariance, radius = 3 sqrt(lambda_max), and visibility =
// in front of the near plane, positive determinant and an opacity-aware tile rectangle that
// touches the grid.  One thread per gaussian; the [n,3] / [n,4] rows a warp reads are contiguous,
// so the loads are coalesced through L1 without a separate SoA copy.
#include "hds_common.cuh"

namespace hds {
namespace {

struct Camera {
    float fx, fy, cx, cy;
    int width, height;
    float near_plane, low_pass, fov_scale;
};

// Rows 0..2 of world_to_camera, read by every thread from the same 48 bytes (broadcast loads
// served by L1), so the pose never needs a host round trip.
struct Pose {
    float m[12];
    __device__ __forceinline__ explicit Pose(const float* __restrict__ p) {
#pragma unroll
        for (int i = 0; i < 12; i++) m[i] = __ldg(p + i);
    }
};

struct Projected {
    float R[3][3], t[3], p[3];
    float z, z_inv, jx, jy;
    bool clamped_x, clamped_y, behind;
    float jw[2][3], M[3][3], T[2][3];
    float a, b, c, det;
};

__device__ __forceinline__ void quat_rot(float w, float x, float y, float z, float r[3][3]) {
    r[0][0] = 1.0f - 2.0f * (y * y + z * z); r[0][1] = 2.0f * (x * y - w * z); r[0][2] = 2.0f * (x * z + w * y);
    r[1][0] = 2.0f * (x * y + w * z); r[1][1] = 1.0f - 2.0f * (x * x + z * z); r[1][2] = 2.0f * (y * z - w * x);
    r[2][0] = 2.0f * (x * z - w * y); r[2][1] = 2.0f * (y * z + w * x); r[2][2] = 1.0f - 2.0f * (x * x + y * y);
}

__device__ __forceinline__ void project_one(const Camera& cam, const Pose& pose, const float mean[3],
                                            const float scale[3], const float q[4], Projected& g) {
#pragma unroll
    for (int i = 0; i < 3; i++) {
#pragma unroll
        for (int j = 0; j < 3; j++) g.R[i][j] = pose.m[i * 4 + j];
        g.t[i] = pose.m[i * 4 + 3];
        g.p[i] = g.R[i][0] * mean[0] + g.R[i][1] * mean[1] + g.R[i][2] * mean[2] + g.t[i];
    }
    g.behind = g.p[2] <= cam.near_plane;
    g.z = fmaxf(g.p[2], cam.near_plane);
    g.z_inv = 1.0f / (g.z + 1e-6f);
    float limit_x = cam.fov_scale * (0.5f * (float)cam.width / cam.fx);
    float limit_y = cam.fov_scale * (0.5f * (float)cam.height / cam.fy);
    float rx = g.p[0] * g.z_inv, ry = g.p[1] * g.z_inv;
    g.clamped_x = fabsf(rx) > limit_x;
    g.clamped_y = fabsf(ry) > limit_y;
    g.jx = fminf(fmaxf(rx, -limit_x), limit_x) * g.z;
    g.jy = fminf(fmaxf(ry, -limit_y), limit_y) * g.z;
    float zz_inv = g.z_inv * g.z_inv;
#pragma unroll
    for (int j = 0; j < 3; j++) {
        g.jw[0][j] = cam.fx * g.z_inv * g.R[0][j] - cam.fx * g.jx * zz_inv * g.R[2][j];
        g.jw[1][j] = cam.fy * g.z_inv * g.R[1][j] - cam.fy * g.jy * zz_inv * g.R[2][j];
    }
    float rot[3][3];
    quat_rot(q[0], q[1], q[2], q[3], rot);
#pragma unroll
    for (int j = 0; j < 3; j++)
#pragma unroll
        for (int k = 0; k < 3; k++) g.M[j][k] = rot[j][k] * scale[k];
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
        for (int k = 0; k < 3; k++) g.T[r][k] = g.jw[r][0] * g.M[0][k] + g.jw[r][1] * g.M[1][k] + g.jw[r][2] * g.M[2][k];
    g.a = g.T[0][0] * g.T[0][0] + g.T[0][1] * g.T[0][1] + g.T[0][2] * g.T[0][2] + cam.low_pass;
    g.b = g.T[0][0] * g.T[1][0] + g.T[0][1] * g.T[1][1] + g.T[0][2] * g.T[1][2];
    g.c = g.T[1][0] * g.T[1][0] + g.T[1][1] * g.T[1][1] + g.T[1][2] * g.T[1][2] + cam.low_pass;
    g.det = g.a * g.c - g.b * g.b;
}

__device__ __forceinline__ void load_row3(const float* p, int i, float out[3]) {
    out[0] = p[3 * i]; out[1] = p[3 * i + 1]; out[2] = p[3 * i + 2];
}

// The model's parameter activations (the reference's utils/gaussian.py:73-98), applied in the kernel
// when the projection takes raw parameters: scale = exp(log_scale), quat = q / max(|q|, 1e-12) with
// |q| summed w, x, y, z in order (torch.nn.functional.normalize), opacity = 1 / (1 + exp(-logit)).
// expf_det rounds like the CPU oracle's exp.
struct Activated {
    float scale[3], q[4], qlen, opacity;
};

__device__ __forceinline__ void activate(const float log_scale[3], const float raw_q[4], float logit, Activated& a) {
#pragma unroll
    for (int k = 0; k < 3; k++) a.scale[k] = expf_det(log_scale[k]);
    const float w = raw_q[0], x = raw_q[1], y = raw_q[2], z = raw_q[3];
    a.qlen = fmaxf(sqrtf(w * w + x * x + y * y + z * z), 1e-12f);
#pragma unroll
    for (int c = 0; c < 4; c++) a.q[c] = raw_q[c] / a.qlen;
    a.opacity = 1.0f / (1.0f + expf_det(-logit));
}

// RAW: scales, quats and opacities hold the raw parameters (log-scales, unnormalised quaternions,
// opacity logits), activated here; the activated opacity is written to opacities_out.
template <bool RAW>
__global__ void __launch_bounds__(256) project_forward_kernel(int n, Camera cam, const float* __restrict__ w2c, const float* __restrict__ means,
                                                              const float* __restrict__ scales, const float* __restrict__ quats,
                                                              const float* __restrict__ opacities, float* __restrict__ means2D,
                                                              float* __restrict__ depths, float* __restrict__ radii,
                                                              float* __restrict__ conics, float* __restrict__ opacities_out) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const Pose pose(w2c);
    float mean[3], scale[3];
    load_row3(means, i, mean);
    load_row3(scales, i, scale);
    float4 q = reinterpret_cast<const float4*>(quats)[i];
    float qa[4] = {q.x, q.y, q.z, q.w};
    float opacity = opacities[i];
    if (RAW) {
        Activated act;
        activate(scale, qa, opacity, act);
#pragma unroll
        for (int k = 0; k < 3; k++) scale[k] = act.scale[k];
#pragma unroll
        for (int c = 0; c < 4; c++) qa[c] = act.q[c];
        opacity = act.opacity;
        opacities_out[i] = opacity;
    }
    Projected g;
    project_one(cam, pose, mean, scale, qa, g);
    float u = cam.fx * g.p[0] / g.z + cam.cx;
    float v = cam.fy * g.p[1] / g.z + cam.cy;
    reinterpret_cast<float2*>(means2D)[i] = make_float2(u, v);
    depths[i] = g.p[2];
    float scale_inv = g.det > 0.0f ? 1.0f / g.det : 1.0f;
    float ca = g.c * scale_inv, cb = -g.b * scale_inv, cc = g.a * scale_inv;
    conics[3 * i] = ca;
    conics[3 * i + 1] = cb;
    conics[3 * i + 2] = cc;
    float trace = g.a + g.c;
    float radius = 3.0f * sqrtf(0.5f * (trace + sqrtf(fmaxf(trace * trace - 4.0f * g.det, 0.0f))));
    int x0, y0, x1, y1;
    bool visible = !g.behind && g.det > 0.0f &&
                   tile_rect(u, v, ca, cb, cc, opacity, tiles_for(cam.width), tiles_for(cam.height), x0, y0, x1, y1);
    radii[i] = visible ? radius : 0.0f;
}

// RAW: as in the forward, the inputs are raw parameters and the gradients go to them (through the
// activations); grad_opacities (may be null: zero) is dL/d(activated opacity), and grad_logits
// receives dL/dlogit.  ACCUMULATE adds every gradient to what its buffer holds.
template <bool RAW, bool ACCUMULATE>
__global__ void __launch_bounds__(256) project_backward_kernel(int n, Camera cam, const float* __restrict__ w2c, const float* __restrict__ grad_means2D,
                                                               const float* __restrict__ grad_conics,
                                                               const float* __restrict__ means, const float* __restrict__ scales,
                                                               const float* __restrict__ quats, float* __restrict__ grad_means,
                                                               float* __restrict__ grad_scales, float* __restrict__ grad_quats,
                                                               const float* __restrict__ logits,
                                                               const float* __restrict__ grad_opacities,
                                                               float* __restrict__ grad_logits) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const Pose pose(w2c);
    float mean[3], scale[3];
    load_row3(means, i, mean);
    load_row3(scales, i, scale);
    float4 q4 = reinterpret_cast<const float4*>(quats)[i];
    float q[4] = {q4.x, q4.y, q4.z, q4.w};
    Activated act;
    if (RAW) {
        activate(scale, q, logits[i], act);
#pragma unroll
        for (int k = 0; k < 3; k++) scale[k] = act.scale[k];
#pragma unroll
        for (int c = 0; c < 4; c++) q[c] = act.q[c];
    }
    Projected g;
    project_one(cam, pose, mean, scale, q, g);

    float g0 = grad_conics[3 * i], g1 = grad_conics[3 * i + 1], g2 = grad_conics[3 * i + 2];
    float da, db, dc;
    if (g.det > 0.0f) {
        float inv = 1.0f / g.det, inv2 = inv * inv;
        da = inv2 * (-g0 * g.c * g.c + g1 * g.b * g.c - g2 * g.b * g.b);
        db = inv2 * (2.0f * g0 * g.b * g.c + 2.0f * g2 * g.a * g.b) - g1 * (inv + 2.0f * g.b * g.b * inv2);
        dc = inv2 * (-g0 * g.b * g.b + g1 * g.a * g.b - g2 * g.a * g.a);
    } else {
        da = g2; db = -g1; dc = g0;
    }
    float dT[2][3];
#pragma unroll
    for (int k = 0; k < 3; k++) {
        dT[0][k] = 2.0f * da * g.T[0][k] + db * g.T[1][k];
        dT[1][k] = 2.0f * dc * g.T[1][k] + db * g.T[0][k];
    }
    float rot[3][3];
    quat_rot(q[0], q[1], q[2], q[3], rot);
    float djw[2][3], drot[3][3], dscale[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int j = 0; j < 3; j++) {
        djw[0][j] = dT[0][0] * g.M[j][0] + dT[0][1] * g.M[j][1] + dT[0][2] * g.M[j][2];
        djw[1][j] = dT[1][0] * g.M[j][0] + dT[1][1] * g.M[j][1] + dT[1][2] * g.M[j][2];
#pragma unroll
        for (int k = 0; k < 3; k++) {
            float dM = g.jw[0][j] * dT[0][k] + g.jw[1][j] * dT[1][k];
            dscale[k] += dM * rot[j][k];
            drot[j][k] = dM * scale[k];
        }
    }
    float w = q[0], x = q[1], y = q[2], z = q[3];
    float4 gq;
    gq.x = 2.0f * (-drot[0][1] * z + drot[0][2] * y + drot[1][0] * z - drot[1][2] * x - drot[2][0] * y + drot[2][1] * x);
    gq.y = 2.0f * (drot[0][1] * y + drot[0][2] * z + drot[1][0] * y - 2.0f * drot[1][1] * x - drot[1][2] * w
                   + drot[2][0] * z + drot[2][1] * w - 2.0f * drot[2][2] * x);
    gq.z = 2.0f * (-2.0f * drot[0][0] * y + drot[0][1] * x + drot[0][2] * w + drot[1][0] * x + drot[1][2] * z
                   - drot[2][0] * w + drot[2][1] * z - 2.0f * drot[2][2] * y);
    gq.w = 2.0f * (-2.0f * drot[0][0] * z - drot[0][1] * w + drot[0][2] * x + drot[1][0] * w - 2.0f * drot[1][1] * z
                   + drot[1][2] * y + drot[2][0] * x + drot[2][1] * y);
    if (RAW) {
        // Through q / |q|: (g - q (q . g)) / |q| above the clamp, g / |q| at it; through exp: times
        // the scale; through the sigmoid: times s (1 - s).
        const float qv[4] = {q[0], q[1], q[2], q[3]};
        const float gv[4] = {gq.x, gq.y, gq.z, gq.w};
        float out[4];
        if (act.qlen > 1e-12f) {
            const float dot = qv[0] * gv[0] + qv[1] * gv[1] + qv[2] * gv[2] + qv[3] * gv[3];
#pragma unroll
            for (int c = 0; c < 4; c++) out[c] = (gv[c] - qv[c] * dot) / act.qlen;
        } else {
#pragma unroll
            for (int c = 0; c < 4; c++) out[c] = gv[c] / act.qlen;
        }
        gq = make_float4(out[0], out[1], out[2], out[3]);
#pragma unroll
        for (int k = 0; k < 3; k++) dscale[k] = dscale[k] * scale[k];
        const float gop = grad_opacities != nullptr ? grad_opacities[i] : 0.0f;
        const float dlogit = gop * (act.opacity * (1.0f - act.opacity));
        grad_logits[i] = ACCUMULATE ? grad_logits[i] + dlogit : dlogit;
    }
    if (ACCUMULATE) {
        const float4 old = reinterpret_cast<const float4*>(grad_quats)[i];
        gq = make_float4(old.x + gq.x, old.y + gq.y, old.z + gq.z, old.w + gq.w);
#pragma unroll
        for (int k = 0; k < 3; k++) dscale[k] = grad_scales[3 * i + k] + dscale[k];
    }
    reinterpret_cast<float4*>(grad_quats)[i] = gq;
#pragma unroll
    for (int k = 0; k < 3; k++) grad_scales[3 * i + k] = dscale[k];

    float zz_inv = g.z_inv * g.z_inv;
    float dz_inv = 0.0f, djx = 0.0f, djy = 0.0f;
#pragma unroll
    for (int j = 0; j < 3; j++) {
        dz_inv += djw[0][j] * (cam.fx * g.R[0][j] - 2.0f * cam.fx * g.jx * g.z_inv * g.R[2][j]);
        dz_inv += djw[1][j] * (cam.fy * g.R[1][j] - 2.0f * cam.fy * g.jy * g.z_inv * g.R[2][j]);
        djx += djw[0][j] * (-cam.fx * zz_inv * g.R[2][j]);
        djy += djw[1][j] * (-cam.fy * zz_inv * g.R[2][j]);
    }
    float dp[3] = {0.0f, 0.0f, 0.0f};
    float dz = 0.0f;
    float rx = g.jx / g.z, ry = g.jy / g.z;
    dz += djx * rx + djy * ry;
    if (!g.clamped_x) { dp[0] += djx * g.z * g.z_inv; dz_inv += djx * g.z * g.p[0]; }
    if (!g.clamped_y) { dp[1] += djy * g.z * g.z_inv; dz_inv += djy * g.z * g.p[1]; }
    float gu = grad_means2D[2 * i], gv = grad_means2D[2 * i + 1];
    dp[0] += gu * cam.fx / g.z;
    dp[1] += gv * cam.fy / g.z;
    dz += -(gu * cam.fx * g.p[0] + gv * cam.fy * g.p[1]) / (g.z * g.z);
    dz += dz_inv * (-zz_inv);
    if (!g.behind) dp[2] += dz;
#pragma unroll
    for (int k = 0; k < 3; k++) {
        const float gm = g.R[0][k] * dp[0] + g.R[1][k] * dp[1] + g.R[2][k] * dp[2];
        grad_means[3 * i + k] = ACCUMULATE ? grad_means[3 * i + k] + gm : gm;
    }
}

bool aligned(const void* p, uintptr_t bytes) { return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0; }

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" int hds_project_forward(int n, const float* means, const float* scales, const float* quats,
                                   const float* opacities, const float* world_to_camera, float fx, float fy, float cx,
                                   float cy, int width, int height, float near_plane, float low_pass, float fov_scale,
                                   float* means2D, float* depths, float* radii, float* conics, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0, HDS_ERR_INVALID, "project_forward: bad sizes n=%d %dx%d", n, width,
                height);
    if (n == 0) return HDS_OK;
    HDS_REQUIRE(aligned(quats, 16) && aligned(means2D, 8), HDS_ERR_INVALID,
                "project_forward: quats must be 16-byte and means2D 8-byte aligned");
    Camera cam{fx, fy, cx, cy, width, height, near_plane, low_pass, fov_scale};
    project_forward_kernel<false><<<(n + 255) / 256, 256, 0, stream>>>(n, cam, world_to_camera, means, scales, quats,
                                                                       opacities, means2D, depths, radii, conics, nullptr);
    HDS_CHECK_LAUNCH("project_forward_kernel");
    return HDS_OK;
}

extern "C" int hds_project_backward(int n, const float* grad_means2D, const float* grad_conics, const float* means,
                                    const float* scales, const float* quats, const float* world_to_camera, float fx,
                                    float fy, float cx, float cy, int width, int height, float near_plane,
                                    float low_pass, float fov_scale, float* grad_means, float* grad_scales,
                                    float* grad_quats, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0, HDS_ERR_INVALID, "project_backward: bad sizes");
    if (n == 0) return HDS_OK;
    HDS_REQUIRE(aligned(quats, 16) && aligned(grad_quats, 16), HDS_ERR_INVALID,
                "project_backward: quats and grad_quats must be 16-byte aligned");
    Camera cam{fx, fy, cx, cy, width, height, near_plane, low_pass, fov_scale};
    project_backward_kernel<false, false><<<(n + 255) / 256, 256, 0, stream>>>(
        n, cam, world_to_camera, grad_means2D, grad_conics, means, scales, quats, grad_means, grad_scales, grad_quats,
        nullptr, nullptr, nullptr);
    HDS_CHECK_LAUNCH("project_backward_kernel");
    return HDS_OK;
}

extern "C" int hds_project_forward_raw(int n, const float* means, const float* log_scales, const float* quats,
                                       const float* opacity_logits, const float* world_to_camera, float fx, float fy,
                                       float cx, float cy, int width, int height, float near_plane, float low_pass,
                                       float fov_scale, float* means2D, float* depths, float* radii, float* conics,
                                       float* opacities, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0, HDS_ERR_INVALID, "project_forward_raw: bad sizes n=%d %dx%d", n,
                width, height);
    if (n == 0) return HDS_OK;
    HDS_REQUIRE(aligned(quats, 16) && aligned(means2D, 8), HDS_ERR_INVALID,
                "project_forward_raw: quats must be 16-byte and means2D 8-byte aligned");
    Camera cam{fx, fy, cx, cy, width, height, near_plane, low_pass, fov_scale};
    project_forward_kernel<true><<<(n + 255) / 256, 256, 0, stream>>>(n, cam, world_to_camera, means, log_scales, quats,
                                                                      opacity_logits, means2D, depths, radii, conics,
                                                                      opacities);
    HDS_CHECK_LAUNCH("project_forward_kernel");
    return HDS_OK;
}

extern "C" int hds_project_backward_raw(int n, const float* grad_means2D, const float* grad_conics,
                                        const float* grad_opacities, const float* means, const float* log_scales,
                                        const float* quats, const float* opacity_logits, const float* world_to_camera,
                                        float fx, float fy, float cx, float cy, int width, int height,
                                        float near_plane, float low_pass, float fov_scale, float* grad_means,
                                        float* grad_log_scales, float* grad_quats, float* grad_opacity_logits,
                                        int accumulate, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0, HDS_ERR_INVALID, "project_backward_raw: bad sizes");
    if (n == 0) return HDS_OK;
    HDS_REQUIRE(aligned(quats, 16) && aligned(grad_quats, 16), HDS_ERR_INVALID,
                "project_backward_raw: quats and grad_quats must be 16-byte aligned");
    Camera cam{fx, fy, cx, cy, width, height, near_plane, low_pass, fov_scale};
    const unsigned blocks = (unsigned)((n + 255) / 256);
    if (accumulate)
        project_backward_kernel<true, true><<<blocks, 256, 0, stream>>>(
            n, cam, world_to_camera, grad_means2D, grad_conics, means, log_scales, quats, grad_means, grad_log_scales,
            grad_quats, opacity_logits, grad_opacities, grad_opacity_logits);
    else
        project_backward_kernel<true, false><<<blocks, 256, 0, stream>>>(
            n, cam, world_to_camera, grad_means2D, grad_conics, means, log_scales, quats, grad_means, grad_log_scales,
            grad_quats, opacity_logits, grad_opacities, grad_opacity_logits);
    HDS_CHECK_LAUNCH("project_backward_kernel");
    return HDS_OK;
}
