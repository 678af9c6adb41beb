// hds_common.cuh -- constants, scalar math and error plumbing shared by every kernel.
//
// The library is compiled with --fmad=false: a*b+c rounds twice unless a kernel writes fmaf()
// itself.  Together with IEEE division/sqrt (no fast math) and the two scalar functions below,
// every forward output rounds exactly like the CPU oracle, which writes the same operations.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>

#include "hds_b200.h"

namespace hds {

// common.cuh:8-16 of the reference.
constexpr int TILE = 16;
constexpr int TILE_PIXELS = TILE * TILE;
constexpr float MIN_ALPHA = 0x1.010102p-8f;  // 1.0f / 255.0f
constexpr float MAX_ALPHA = 0.99f;
constexpr float MIN_T = 1e-4f;
constexpr unsigned FULL_MASK = 0xffffffffu;

__host__ __device__ inline int tiles_for(int pixels) { return (pixels + TILE - 1) / TILE; }

// exp(x): n = rint(x log2 e), r = x - n ln2 (Cody-Waite split), e^r by its Taylor series to r^7/7!,
// scaled by 2^n.  Identical operations to oracle_expf in the CPU restatement.
__device__ __forceinline__ float expf_det(float x) {
    x = fminf(fmaxf(x, -87.0f), 88.0f);
    float t = __fmul_rn(x, 0x1.715476p+0f);
    float n = rintf(t);
    float r = fmaf(-n, 0x1.62e4p-1f, x);
    r = fmaf(-n, 0x1.7f7d1cp-20f, r);
    float p = 0x1.a01a02p-13f;
    p = fmaf(p, r, 0x1.6c16c2p-10f);
    p = fmaf(p, r, 0x1.111112p-7f);
    p = fmaf(p, r, 0x1.555556p-5f);
    p = fmaf(p, r, 0x1.555556p-3f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int e = __float2int_rn(n) + 127;
    return __fmul_rn(p, __int_as_float(e << 23));
}

// log(y) for finite normal y > 0 by the atanh series; identical to oracle_logf.
__device__ __forceinline__ float logf_det(float y) {
    uint32_t bits = __float_as_uint(y);
    int e = (int)((bits >> 23) & 0xffu) - 127;
    float m = __uint_as_float((bits & 0x007fffffu) | 0x3f800000u);
    if (m > 0x1.6a09e6p+0f) {
        m = __fmul_rn(m, 0.5f);
        e = e + 1;
    }
    float s = __fdiv_rn(__fsub_rn(m, 1.0f), __fadd_rn(m, 1.0f));
    float s2 = __fmul_rn(s, s);
    float q = 0x1.c71c72p-4f;
    q = fmaf(q, s2, 0x1.24924ap-3f);
    q = fmaf(q, s2, 0x1.99999ap-3f);
    q = fmaf(q, s2, 0x1.555556p-2f);
    q = fmaf(q, s2, 1.0f);
    float lm = __fmul_rn(__fmul_rn(2.0f, s), q);
    float fe = (float)e;
    return fmaf(fe, 0x1.62e4p-1f, fmaf(fe, 0x1.7f7d1cp-20f, lm));
}

// common.cuh:49-65 of the reference (alpha_extent + tile_rect): the opacity-aware ellipse box,
// as an inclusive tile rectangle.  Clamped in float before the int conversion so NaN or huge
// coordinates are rejected.  Identical to oracle_tile_rect.  The grid is tile rows
// [row0, row0 + tiles_y) of the full image (row0 = 0: the whole image); (u, v) are full-image pixel
// coordinates and the returned rows count from row0, so a band of rows gets exactly the tiles the
// full image's rectangle has there.
__device__ __forceinline__ bool tile_rect(float u, float v, float a, float b, float c, float opacity, int tiles_x,
                                          int row0, int tiles_y, int& x0, int& y0, int& x1, int& y1) {
    if (!(opacity > MIN_ALPHA)) return false;
    float k = __fsqrt_rn(__fmul_rn(2.0f, logf_det(__fdiv_rn(opacity, MIN_ALPHA))));
    float det = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, b));
    float ex = __fmul_rn(k, __fsqrt_rn(__fdiv_rn(c, det)));
    float ey = __fmul_rn(k, __fsqrt_rn(__fdiv_rn(a, det)));
    float lx = floorf(__fdiv_rn(__fsub_rn(u, ex), 16.0f)), hx = floorf(__fdiv_rn(__fadd_rn(u, ex), 16.0f));
    float ly = floorf(__fdiv_rn(__fsub_rn(v, ey), 16.0f)), hy = floorf(__fdiv_rn(__fadd_rn(v, ey), 16.0f));
    float fx0 = fmaxf(lx, 0.0f), fx1 = fminf(hx, (float)(tiles_x - 1));
    float fy0 = fmaxf(ly, (float)row0), fy1 = fminf(hy, (float)(row0 + tiles_y - 1));
    if (!(fx1 >= fx0 && fy1 >= fy0)) return false;
    x0 = (int)fx0; x1 = (int)fx1; y0 = (int)fy0 - row0; y1 = (int)fy1 - row0;
    return true;
}

// Reads and clears the feature backward kernel's device status (render_features_bwd.cu); the
// copies are queued on `stream`.
int read_and_clear_backward_status(int* status, cudaStream_t stream);

// Lane of the (n+1)-th set bit of mask (n >= 0, fewer than popc(mask)).
__device__ __forceinline__ int nth_set_bit(unsigned mask, int n) {
    for (int i = 0; i < n; i++) mask &= mask - 1;
    return __ffs(mask) - 1;
}

// The per-pair opacity term of every blend: mahalanobis distance of the pixel centre under the
// conic, G = exp(-m/2), raw alpha = opacity * G (forward.cu:197-208).  Same order as the oracle.
// The backward walks use it too, so every pair's alpha -- and which side of the MIN_ALPHA cutoff it
// falls on -- is bit-identical in the forward, the backward and the oracle.
struct PairAlpha {
    float dx, dy, G, raw;
};

__device__ __forceinline__ PairAlpha pair_alpha(float px, float py, float mx, float my, float a, float b, float c,
                                                float opacity) {
    PairAlpha r;
    r.dx = __fsub_rn(px, mx);
    r.dy = __fsub_rn(py, my);
    float t1 = fmaf(b, r.dy, __fmul_rn(a, r.dx));
    float t2 = fmaf(c, r.dy, __fmul_rn(b, r.dx));
    float maha = fmaf(r.dy, t2, __fmul_rn(r.dx, t1));
    r.G = expf_det(__fmul_rn(-0.5f, maha));
    r.raw = __fmul_rn(opacity, r.G);
    return r;
}

// Conservative half-widths of the box where alpha can reach MIN_ALPHA: the binning extent widened
// by 0.1% + 0.01 px so rounding never culls a pair the walk would blend (the reference's
// features.cu:8-17).  Opacity <= MIN_ALPHA never blends (negative extent: hits nothing); a
// degenerate conic (NaN extent) hits everything.
__device__ __forceinline__ float2 cull_extent(float a, float b, float c, float opacity) {
    if (!(opacity > MIN_ALPHA)) return make_float2(-1e30f, -1e30f);
    float k = sqrtf(2.0f * logf_det(opacity / MIN_ALPHA));
    float det = a * c - b * b;
    float ex = k * sqrtf(c / det) * 1.001f + 0.01f;
    float ey = k * sqrtf(a / det) * 1.001f + 0.01f;
    if (!(ex >= 0.0f)) ex = 1e30f;
    if (!(ey >= 0.0f)) ey = 1e30f;
    return make_float2(ex, ey);
}

// cull_extent with approximate reciprocal and log: their errors (~1e-6 relative) are far inside
// the box's 0.1% + 0.01 px widening, so the box stays conservative.  A degenerate conic (det <= 0)
// still hits everything.
__device__ __forceinline__ float2 cull_extent_fast(float a, float b, float c, float opacity) {
    if (!(opacity > MIN_ALPHA)) return make_float2(-1e30f, -1e30f);
    const float k = sqrtf(2.0f * __logf(opacity * (1.0f / MIN_ALPHA)));
    const float inv_det = __fdividef(1.0f, a * c - b * b);
    float ex = k * sqrtf(c * inv_det) * 1.001f + 0.01f;
    float ey = k * sqrtf(a * inv_det) * 1.001f + 0.01f;
    if (!(ex >= 0.0f)) ex = 1e30f;
    if (!(ey >= 0.0f)) ey = 1e30f;
    return make_float2(ex, ey);
}

// Does the box mean +- extent touch the pixel-centre rectangle [x0, x1] x [y0, y1]?
__device__ __forceinline__ bool box_hits(float2 m, float2 e, float x0, float x1, float y0, float y1) {
    return m.x + e.x >= x0 && m.x - e.x <= x1 && m.y + e.y >= y0 && m.y - e.y <= y1;
}

// ---------------------------------------------------------------------------------------------
// host-side error plumbing
// ---------------------------------------------------------------------------------------------
void set_error(const char* fmt, ...);
void clear_error();
void note_launches(int n);  // counts kernel launches for hds_launch_count()

inline int cuda_fail(cudaError_t err, const char* what) {
    set_error("CUDA error in %s: %s", what, cudaGetErrorString(err));
    return HDS_ERR_CUDA;
}

}  // namespace hds

// After exactly one kernel launch: counts it and turns a launch error into HDS_ERR_CUDA.
#define HDS_CHECK_LAUNCH(name)                                   \
    do {                                                         \
        hds::note_launches(1);                                   \
        cudaError_t err__ = cudaGetLastError();                  \
        if (err__ != cudaSuccess) return hds::cuda_fail(err__, name); \
    } while (0)

#define HDS_CHECK_CUDA(call)                                     \
    do {                                                         \
        cudaError_t err__ = (call);                              \
        if (err__ != cudaSuccess) return hds::cuda_fail(err__, #call); \
    } while (0)

#define HDS_REQUIRE(cond, code, ...)   \
    do {                               \
        if (!(cond)) {                 \
            hds::set_error(__VA_ARGS__); \
            return (code);             \
        }                              \
    } while (0)
