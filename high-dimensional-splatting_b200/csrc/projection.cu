// projection.cu -- EWA projection of 3-D gaussians into the image plane, and its analytic backward.
//
// Semantics of the reference's projection.cu:36-197 (project, project_forward, project_backward):
// the camera-space point p = R m + t; depth z = max(p_z, near) with zi = 1 / (z + 1e-6); the
// perspective Jacobian taken at the tangents p_x zi, p_y zi clamped to fov_scale * half the field of
// view; the 2-D covariance J W Rq S^2 Rq^T W^T J^T + low_pass I; conic = its inverse (the raw
// (c, -b, a) when the determinant is not positive); radius = 3 sqrt(lambda_max); visibility = in
// front of the near plane, positive determinant, and an opacity-aware tile rectangle on the grid.
//
// Formulation used here (the CPU oracle's oracle_project_* states the same operations in the same
// order, so both round identically):
//   A = J W, row r: A_r = e_r (R_r - kappa_r R_2), e_r = f_r zi, kappa_r = (tan_r z) zi
//   Rq = (1 - 2|v|^2) I + 2 (v v^T + w [v]x)       (q = (w, v), not renormalised)
//   B = A Rq, T = B diag(s), Sigma = T T^T + low_pass I = [[a, b], [b, c]]
// and the backward is the chain rule through those factors in matrix form:
//   dSigma = -Q G Q (Q the conic matrix, G the symmetric conic gradient, off-diagonals g_b / 2);
//   dT = 2 dSigma_sym T;  ds_k = <dT_k, B_k>;  dB = dT diag(s);  dA = dB Rq^T;  dRq = A^T dB;
//   dw = 2 v . ax(dRq), dv = 2 ((dRq + dRq^T) v - 2 tr(dRq) v + w ax(dRq)) with ax(D) the axial
//   vector (D21 - D12, D02 - D20, D10 - D01); then (sigma_r, rho_r) = (dA_r . R_r, dA_r . R_2) carry
//   the gradient to e_r and kappa_r, and from there to zi, z, the tangents and p.
//
// Memory: one thread per gaussian, 128 gaussians per block.  The block's [128, 3] rows (means,
// scales, conics and their gradients) move as 96 whole float4s through shared memory, quaternions
// as one float4 per thread, so every global access is a 16-byte, fully coalesced transfer; blocks
// that are partial or whose rows are not 16-byte aligned fall back to element accesses.
#include "hds_common.cuh"

namespace hds {
namespace {

constexpr int PBLOCK = 128;
constexpr int ROW3_F4 = PBLOCK * 3 / 4;  // float4s of a block's [PBLOCK, 3] rows
static_assert(PBLOCK * 3 % 4 == 0 && ROW3_F4 <= PBLOCK, "a block's [PBLOCK, 3] rows must be whole float4s");

struct Camera {
    float fx, fy, cx, cy;
    int width, height;
    float near_plane, low_pass, fov_scale;
};

// Rows 0..2 of world_to_camera, read by every thread from the same 48 bytes (broadcast loads served
// by L1), so the pose never needs a host round trip.
struct Pose {
    float R[3][3], t[3];
    __device__ __forceinline__ explicit Pose(const float* __restrict__ w2c) {
#pragma unroll
        for (int i = 0; i < 3; i++) {
#pragma unroll
            for (int j = 0; j < 3; j++) R[i][j] = __ldg(w2c + 4 * i + j);
            t[i] = __ldg(w2c + 4 * i + 3);
        }
    }
};

// Everything the forward forms and the backward walks back through.
struct Splat {
    float p[3], z, zi;
    float tan[2];
    bool clamped[2], behind;
    float e[2], kappa[2];
    float A[2][3], Rq[3][3], B[2][3], T[2][3];
    float a, b, c, det;
};

__device__ __forceinline__ void splat_forward(const Camera& cam, const Pose& pose, const float m[3],
                                              const float s[3], const float q[4], Splat& g) {
#pragma unroll
    for (int i = 0; i < 3; i++)
        g.p[i] = pose.R[i][0] * m[0] + pose.R[i][1] * m[1] + pose.R[i][2] * m[2] + pose.t[i];
    g.behind = g.p[2] <= cam.near_plane;
    g.z = fmaxf(g.p[2], cam.near_plane);
    g.zi = 1.0f / (g.z + 1e-6f);
    const float lim[2] = {cam.fov_scale * (0.5f * (float)cam.width / cam.fx),
                          cam.fov_scale * (0.5f * (float)cam.height / cam.fy)};
    const float f[2] = {cam.fx, cam.fy};
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const float ratio = g.p[r] * g.zi;
        g.clamped[r] = fabsf(ratio) > lim[r];
        g.tan[r] = fminf(fmaxf(ratio, -lim[r]), lim[r]);
        g.e[r] = f[r] * g.zi;
        g.kappa[r] = (g.tan[r] * g.z) * g.zi;
#pragma unroll
        for (int j = 0; j < 3; j++) g.A[r][j] = g.e[r] * (pose.R[r][j] - g.kappa[r] * pose.R[2][j]);
    }
    const float w = q[0], x = q[1], y = q[2], zq = q[3];
    const float d = 1.0f - 2.0f * (x * x + y * y + zq * zq);
    g.Rq[0][0] = d + 2.0f * (x * x);
    g.Rq[0][1] = 2.0f * (x * y - w * zq);
    g.Rq[0][2] = 2.0f * (x * zq + w * y);
    g.Rq[1][0] = 2.0f * (y * x + w * zq);
    g.Rq[1][1] = d + 2.0f * (y * y);
    g.Rq[1][2] = 2.0f * (y * zq - w * x);
    g.Rq[2][0] = 2.0f * (zq * x - w * y);
    g.Rq[2][1] = 2.0f * (zq * y + w * x);
    g.Rq[2][2] = d + 2.0f * (zq * zq);
#pragma unroll
    for (int r = 0; r < 2; r++)
#pragma unroll
        for (int k = 0; k < 3; k++) {
            g.B[r][k] = g.A[r][0] * g.Rq[0][k] + g.A[r][1] * g.Rq[1][k] + g.A[r][2] * g.Rq[2][k];
            g.T[r][k] = g.B[r][k] * s[k];
        }
    g.a = g.T[0][0] * g.T[0][0] + g.T[0][1] * g.T[0][1] + g.T[0][2] * g.T[0][2] + cam.low_pass;
    g.b = g.T[0][0] * g.T[1][0] + g.T[0][1] * g.T[1][1] + g.T[0][2] * g.T[1][2];
    g.c = g.T[1][0] * g.T[1][0] + g.T[1][1] * g.T[1][1] + g.T[1][2] * g.T[1][2] + cam.low_pass;
    g.det = g.a * g.c - g.b * g.b;
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
    a.qlen = fmaxf(sqrtf(raw_q[0] * raw_q[0] + raw_q[1] * raw_q[1] + raw_q[2] * raw_q[2] + raw_q[3] * raw_q[3]),
                   1e-12f);
#pragma unroll
    for (int c = 0; c < 4; c++) a.q[c] = raw_q[c] / a.qlen;
    a.opacity = 1.0f / (1.0f + expf_det(-logit));
}

__device__ __forceinline__ bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// A block's [count, 3] slice of src (gaussians first..first+count) into s[3 * i + k]: 96 float4 loads
// when the block is whole and the rows are 16-byte aligned, element loads otherwise.  READ_ONLY
// inputs go through the non-coherent read-only path; buffers the kernel later writes do not.
template <bool READ_ONLY = true>
__device__ __forceinline__ void stage3(float* s, const float* src, int first, int count) {
    const float* base = src + 3 * (size_t)first;
    if (count == PBLOCK && aligned16(base)) {
        if (threadIdx.x < ROW3_F4) {
            const float4* b4 = reinterpret_cast<const float4*>(base) + threadIdx.x;
            reinterpret_cast<float4*>(s)[threadIdx.x] = READ_ONLY ? __ldg(b4) : *b4;
        }
    } else {
        for (int e = threadIdx.x; e < 3 * count; e += PBLOCK) s[e] = READ_ONLY ? __ldg(base + e) : base[e];
    }
}

// The reverse of stage3: s[3 * i + k] out to the block's slice of dst.
__device__ __forceinline__ void unstage3(float* __restrict__ dst, const float* s, int first, int count) {
    float* base = dst + 3 * (size_t)first;
    if (count == PBLOCK && aligned16(base)) {
        if (threadIdx.x < ROW3_F4) reinterpret_cast<float4*>(base)[threadIdx.x] = reinterpret_cast<const float4*>(s)[threadIdx.x];
    } else {
        for (int e = threadIdx.x; e < 3 * count; e += PBLOCK) base[e] = s[e];
    }
}

// RAW: scales, quats and opacities hold the raw parameters (log-scales, unnormalised quaternions,
// opacity logits), activated here; the activated opacity is written to opacities_out.
template <bool RAW>
__global__ void __launch_bounds__(PBLOCK) project_forward_kernel(
    int n, Camera cam, const float* __restrict__ w2c, const float* __restrict__ means,
    const float* __restrict__ scales, const float* __restrict__ quats, const float* __restrict__ opacities,
    float* __restrict__ means2D, float* __restrict__ depths, float* __restrict__ radii, float* __restrict__ conics,
    float* __restrict__ opacities_out) {
    __shared__ __align__(16) float s_mean[3 * PBLOCK], s_scale[3 * PBLOCK];
    const int first = blockIdx.x * PBLOCK, count = min(PBLOCK, n - first);
    const int t = threadIdx.x, i = first + t;
    stage3(s_mean, means, first, count);
    stage3(s_scale, scales, first, count);
    float4 q4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float opacity = 0.0f;
    if (t < count) {
        q4 = __ldg(reinterpret_cast<const float4*>(quats) + i);
        opacity = __ldg(opacities + i);
    }
    const Pose pose(w2c);
    __syncthreads();
    // s_mean is dead once read; the conics go out through it.
    float m[3], s[3], q[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
    for (int k = 0; k < 3; k++) {
        m[k] = s_mean[3 * t + k];
        s[k] = s_scale[3 * t + k];
    }
    __syncthreads();
    if (t < count) {
        if (RAW) {
            Activated act;
            activate(s, q, opacity, act);
#pragma unroll
            for (int k = 0; k < 3; k++) s[k] = act.scale[k];
#pragma unroll
            for (int c = 0; c < 4; c++) q[c] = act.q[c];
            opacity = act.opacity;
            opacities_out[i] = opacity;
        }
        Splat g;
        splat_forward(cam, pose, m, s, q, g);
        const float inv = g.det > 0.0f ? 1.0f / g.det : 1.0f;
        const float ca = g.c * inv, cb = -g.b * inv, cc = g.a * inv;
        s_mean[3 * t] = ca;
        s_mean[3 * t + 1] = cb;
        s_mean[3 * t + 2] = cc;
        const float u = cam.fx * (g.p[0] / g.z) + cam.cx;
        const float v = cam.fy * (g.p[1] / g.z) + cam.cy;
        reinterpret_cast<float2*>(means2D)[i] = make_float2(u, v);
        depths[i] = g.p[2];
        const float mid = 0.5f * (g.a + g.c);
        const float lambda = mid + sqrtf(fmaxf(mid * mid - g.det, 0.0f));
        int x0, y0, x1, y1;
        const bool visible = !g.behind && g.det > 0.0f &&
                             tile_rect(u, v, ca, cb, cc, opacity, tiles_for(cam.width), 0, tiles_for(cam.height),
                                       x0, y0, x1, y1);
        radii[i] = visible ? 3.0f * sqrtf(lambda) : 0.0f;
    }
    __syncthreads();
    unstage3(conics, s_mean, first, count);
}

// dL/dSigma (da, db, dc for a, b, c) from dL/dconic (g0, g1, g2 for the stored c/det, -b/det, a/det):
// -Q G Q with G = [[g0, g1/2], [g1/2, g2]]; the raw (c, -b, a) when det <= 0.
__device__ __forceinline__ void covariance_grad(const Splat& g, float g0, float g1, float g2, float& da, float& db,
                                                float& dc) {
    if (g.det > 0.0f) {
        const float inv = 1.0f / g.det;
        const float q00 = g.c * inv, q01 = -g.b * inv, q11 = g.a * inv;
        const float hg = 0.5f * g1;
        const float h00 = g0 * q00 + hg * q01, h01 = g0 * q01 + hg * q11;
        const float h10 = hg * q00 + g2 * q01, h11 = hg * q01 + g2 * q11;
        da = -(q00 * h00 + q01 * h10);
        db = -2.0f * (q00 * h01 + q01 * h11);
        dc = -(q01 * h01 + q11 * h11);
    } else {
        da = g2;
        db = -g1;
        dc = g0;
    }
}

// RAW: as in the forward, the inputs are raw parameters and the gradients go to them (through the
// activations); grad_opacities (may be null: zero) is dL/d(activated opacity), and grad_logits
// receives dL/dlogit.  ACCUMULATE adds every gradient to what its buffer holds.
template <bool RAW, bool ACCUMULATE>
__global__ void __launch_bounds__(PBLOCK) project_backward_kernel(
    int n, Camera cam, const float* __restrict__ w2c, const float* __restrict__ grad_means2D,
    const float* __restrict__ grad_conics, const float* __restrict__ means, const float* __restrict__ scales,
    const float* __restrict__ quats, float* __restrict__ grad_means, float* __restrict__ grad_scales,
    float* __restrict__ grad_quats, const float* __restrict__ logits, const float* __restrict__ grad_opacities,
    float* __restrict__ grad_logits) {
    // With ACCUMULATE the buffers' old rows are staged too, in the same memory phase as the inputs.
    constexpr int ACC_ROWS = ACCUMULATE ? 3 * PBLOCK : 4;
    __shared__ __align__(16) float s_mean[3 * PBLOCK], s_scale[3 * PBLOCK], s_gcon[3 * PBLOCK];
    __shared__ __align__(16) float s_gm_old[ACC_ROWS], s_gs_old[ACC_ROWS];
    const int first = blockIdx.x * PBLOCK, count = min(PBLOCK, n - first);
    const int t = threadIdx.x, i = first + t;
    stage3(s_mean, means, first, count);
    stage3(s_scale, scales, first, count);
    stage3(s_gcon, grad_conics, first, count);
    if (ACCUMULATE) {
        stage3<false>(s_gm_old, grad_means, first, count);
        stage3<false>(s_gs_old, grad_scales, first, count);
    }
    float4 q4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    float2 gm2 = make_float2(0.0f, 0.0f);
    float logit = 0.0f, gop = 0.0f;
    if (t < count) {
        q4 = __ldg(reinterpret_cast<const float4*>(quats) + i);
        gm2 = __ldg(reinterpret_cast<const float2*>(grad_means2D) + i);
        if (RAW) {
            logit = __ldg(logits + i);
            gop = grad_opacities != nullptr ? __ldg(grad_opacities + i) : 0.0f;
        }
    }
    const Pose pose(w2c);
    __syncthreads();
    float m[3], s[3], gc[3], q[4] = {q4.x, q4.y, q4.z, q4.w};
#pragma unroll
    for (int k = 0; k < 3; k++) {
        m[k] = s_mean[3 * t + k];
        s[k] = s_scale[3 * t + k];
        gc[k] = s_gcon[3 * t + k];
    }
    if (t < count) {
        Activated act;
        if (RAW) {
            activate(s, q, logit, act);
#pragma unroll
            for (int k = 0; k < 3; k++) s[k] = act.scale[k];
#pragma unroll
            for (int c = 0; c < 4; c++) q[c] = act.q[c];
        }
        Splat g;
        splat_forward(cam, pose, m, s, q, g);

        float da, db, dc;
        covariance_grad(g, gc[0], gc[1], gc[2], da, db, dc);
        float dT[2][3], ds[3], dB[2][3];
#pragma unroll
        for (int k = 0; k < 3; k++) {
            dT[0][k] = 2.0f * da * g.T[0][k] + db * g.T[1][k];
            dT[1][k] = db * g.T[0][k] + 2.0f * dc * g.T[1][k];
            ds[k] = dT[0][k] * g.B[0][k] + dT[1][k] * g.B[1][k];
            dB[0][k] = dT[0][k] * s[k];
            dB[1][k] = dT[1][k] * s[k];
        }
        float dA[2][3], D[3][3];
#pragma unroll
        for (int j = 0; j < 3; j++) {
#pragma unroll
            for (int r = 0; r < 2; r++) dA[r][j] = dB[r][0] * g.Rq[j][0] + dB[r][1] * g.Rq[j][1] + dB[r][2] * g.Rq[j][2];
#pragma unroll
            for (int k = 0; k < 3; k++) D[j][k] = g.A[0][j] * dB[0][k] + g.A[1][j] * dB[1][k];
        }
        // dL/dq through Rq = (1 - 2|v|^2) I + 2 (v v^T + w [v]x).
        const float w = q[0], x = q[1], y = q[2], zq = q[3];
        const float ax = D[2][1] - D[1][2], ay = D[0][2] - D[2][0], az = D[1][0] - D[0][1];
        const float tr2 = 2.0f * (D[0][0] + D[1][1] + D[2][2]);
        const float svx = 2.0f * D[0][0] * x + (D[0][1] + D[1][0]) * y + (D[0][2] + D[2][0]) * zq;
        const float svy = (D[0][1] + D[1][0]) * x + 2.0f * D[1][1] * y + (D[1][2] + D[2][1]) * zq;
        const float svz = (D[0][2] + D[2][0]) * x + (D[1][2] + D[2][1]) * y + 2.0f * D[2][2] * zq;
        float gq[4];
        gq[0] = 2.0f * (ax * x + ay * y + az * zq);
        gq[1] = 2.0f * (svx - tr2 * x + w * ax);
        gq[2] = 2.0f * (svy - tr2 * y + w * ay);
        gq[3] = 2.0f * (svz - tr2 * zq + w * az);

        // From A_r = e_r (R_r - kappa_r R_2) back to the camera-space point.
        const float f[2] = {cam.fx, cam.fy};
        float dzi = 0.0f, dz = 0.0f, dp[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const float sigma = dA[r][0] * pose.R[r][0] + dA[r][1] * pose.R[r][1] + dA[r][2] * pose.R[r][2];
            const float rho = dA[r][0] * pose.R[2][0] + dA[r][1] * pose.R[2][1] + dA[r][2] * pose.R[2][2];
            const float de = sigma - g.kappa[r] * rho;
            const float dkappa = -g.e[r] * rho;
            dzi += f[r] * de + dkappa * (g.tan[r] * g.z);
            dz += dkappa * (g.tan[r] * g.zi);
            if (!g.clamped[r]) {
                const float dtan = dkappa * (g.z * g.zi);
                dp[r] += dtan * g.zi;
                dzi += dtan * g.p[r];
            }
        }
        // means2D = f (p / z) + c.
        const float gm[2] = {gm2.x, gm2.y};
#pragma unroll
        for (int r = 0; r < 2; r++) {
            const float dratio = gm[r] * f[r];
            dp[r] += dratio / g.z;
            dz -= dratio * (g.p[r] / g.z) / g.z;
        }
        dz += dzi * -(g.zi * g.zi);
        if (!g.behind) dp[2] += dz;

        if (RAW) {
            // Through q / |q|: (g - q (q . g)) / |q| above the clamp, g / |q| at it; through exp: times
            // the scale; through the sigmoid: times s (1 - s).
            if (act.qlen > 1e-12f) {
                const float dot = q[0] * gq[0] + q[1] * gq[1] + q[2] * gq[2] + q[3] * gq[3];
#pragma unroll
                for (int c = 0; c < 4; c++) gq[c] = (gq[c] - q[c] * dot) / act.qlen;
            } else {
#pragma unroll
                for (int c = 0; c < 4; c++) gq[c] = gq[c] / act.qlen;
            }
#pragma unroll
            for (int k = 0; k < 3; k++) ds[k] = ds[k] * s[k];
            const float dlogit = gop * (act.opacity * (1.0f - act.opacity));
            grad_logits[i] = ACCUMULATE ? grad_logits[i] + dlogit : dlogit;
        }
        float4 out_q = make_float4(gq[0], gq[1], gq[2], gq[3]);
        if (ACCUMULATE) {
            const float4 old = reinterpret_cast<const float4*>(grad_quats)[i];
            out_q = make_float4(old.x + out_q.x, old.y + out_q.y, old.z + out_q.z, old.w + out_q.w);
        }
        reinterpret_cast<float4*>(grad_quats)[i] = out_q;
#pragma unroll
        for (int k = 0; k < 3; k++) {
            const float gmk = pose.R[0][k] * dp[0] + pose.R[1][k] * dp[1] + pose.R[2][k] * dp[2];
            s_mean[3 * t + k] = ACCUMULATE ? s_gm_old[3 * t + k] + gmk : gmk;
            s_scale[3 * t + k] = ACCUMULATE ? s_gs_old[3 * t + k] + ds[k] : ds[k];
        }
    }
    __syncthreads();
    unstage3(grad_means, s_mean, first, count);
    unstage3(grad_scales, s_scale, first, count);
}

bool aligned(const void* p, uintptr_t bytes) { return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0; }

unsigned blocks_for(int n) { return (unsigned)((n + PBLOCK - 1) / PBLOCK); }

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
    project_forward_kernel<false><<<blocks_for(n), PBLOCK, 0, stream>>>(n, cam, world_to_camera, means, scales, quats,
                                                                        opacities, means2D, depths, radii, conics,
                                                                        nullptr);
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
    HDS_REQUIRE(aligned(quats, 16) && aligned(grad_quats, 16) && aligned(grad_means2D, 8), HDS_ERR_INVALID,
                "project_backward: quats and grad_quats must be 16-byte and grad_means2D 8-byte aligned");
    Camera cam{fx, fy, cx, cy, width, height, near_plane, low_pass, fov_scale};
    project_backward_kernel<false, false><<<blocks_for(n), PBLOCK, 0, stream>>>(
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
    project_forward_kernel<true><<<blocks_for(n), PBLOCK, 0, stream>>>(n, cam, world_to_camera, means, log_scales,
                                                                       quats, opacity_logits, means2D, depths, radii,
                                                                       conics, opacities);
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
    HDS_REQUIRE(aligned(quats, 16) && aligned(grad_quats, 16) && aligned(grad_means2D, 8), HDS_ERR_INVALID,
                "project_backward_raw: quats and grad_quats must be 16-byte and grad_means2D 8-byte aligned");
    Camera cam{fx, fy, cx, cy, width, height, near_plane, low_pass, fov_scale};
    if (accumulate)
        project_backward_kernel<true, true><<<blocks_for(n), PBLOCK, 0, stream>>>(
            n, cam, world_to_camera, grad_means2D, grad_conics, means, log_scales, quats, grad_means, grad_log_scales,
            grad_quats, opacity_logits, grad_opacities, grad_opacity_logits);
    else
        project_backward_kernel<true, false><<<blocks_for(n), PBLOCK, 0, stream>>>(
            n, cam, world_to_camera, grad_means2D, grad_conics, means, log_scales, quats, grad_means, grad_log_scales,
            grad_quats, opacity_logits, grad_opacities, grad_opacity_logits);
    HDS_CHECK_LAUNCH("project_backward_kernel");
    return HDS_OK;
}
