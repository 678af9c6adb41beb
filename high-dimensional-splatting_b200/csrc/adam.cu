// adam.cu -- one Adam step over every gaussian parameter at once: the flat fp32 buffers that hold all
// parameters of a model back to back, their two moments, and the flat gradient bucket the backward
// passes accumulate into.
//
// This is the optimizer step of the reference's training loop (main.py:194, torch.optim.Adam with
// fused=True over one parameter group per tensor), as one memory-bound kernel: each element reads its
// parameter, two moments and gradient and writes the first three back (28 bytes), the group it
// belongs to -- and so its learning rate -- given by a small table of segment ends.  The element
// update is the reference's own Adam form (sh.cu:90-102): m += (1 - b1) (g - m),
// v = b2 v + (1 - b2) g g, p -= (lr / (1 - b1^t)) m / (sqrt(v) / sqrt(1 - b2^t) + eps).
//
// Layout and traffic: 16-byte loads and stores of whole float4s (grid-stride over float4 chunks, four
// chunks in flight per thread), with the streaming cache hint (each byte is touched once); a chunk
// that straddles two segments, or the tail of a length that is not a multiple of four, goes element by
// element.  Unaligned buffers take the element path throughout.
#include <algorithm>

#include "hds_common.cuh"

namespace hds {
namespace {

struct AdamTable {
    int segments;
    int64_t end[HDS_ADAM_MAX_SEGMENTS];  // exclusive end of segment s; end[segments - 1] = n
    float step_size[HDS_ADAM_MAX_SEGMENTS];  // lr_s / (1 - beta1^t)
    float bc2_sqrt, beta2, one_minus_beta1, one_minus_beta2, eps;
};

__device__ __forceinline__ int segment_of(const AdamTable& t, int64_t i) {
    int s = 0;
    while (s < t.segments - 1 && i >= t.end[s]) s++;
    return s;
}

__device__ __forceinline__ void adam_one(float& p, float& m, float& v, float g, float step_size, const AdamTable& t) {
    const float mt = m + t.one_minus_beta1 * (g - m);
    const float vt = t.beta2 * v + t.one_minus_beta2 * g * g;
    m = mt;
    v = vt;
    p = p - step_size * mt / (sqrtf(vt) / t.bc2_sqrt + t.eps);
}

constexpr int ADAM_THREADS = 256;
constexpr int ADAM_UNROLL = 4;

__global__ void __launch_bounds__(ADAM_THREADS) adam_flat_kernel(int64_t n, float* __restrict__ params,
                                                                 float* __restrict__ exp_avg,
                                                                 float* __restrict__ exp_avg_sq,
                                                                 const float* __restrict__ grads, AdamTable t,
                                                                 int vector) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vector) {
        const int64_t chunks = n / 4;
        float4* p4 = reinterpret_cast<float4*>(params);
        float4* m4 = reinterpret_cast<float4*>(exp_avg);
        float4* v4 = reinterpret_cast<float4*>(exp_avg_sq);
        const float4* g4 = reinterpret_cast<const float4*>(grads);
        for (int64_t c0 = tid; c0 < chunks; c0 += stride * ADAM_UNROLL) {
            float4 p[ADAM_UNROLL], m[ADAM_UNROLL], v[ADAM_UNROLL], g[ADAM_UNROLL];
#pragma unroll
            for (int u = 0; u < ADAM_UNROLL; u++) {
                const int64_t c = c0 + u * stride;
                if (c < chunks) {
                    p[u] = __ldcs(p4 + c);
                    m[u] = __ldcs(m4 + c);
                    v[u] = __ldcs(v4 + c);
                    g[u] = __ldcs(g4 + c);
                }
            }
#pragma unroll
            for (int u = 0; u < ADAM_UNROLL; u++) {
                const int64_t c = c0 + u * stride;
                if (c >= chunks) continue;
                const int64_t e = 4 * c;
                const int s0 = segment_of(t, e), s3 = segment_of(t, e + 3);
                if (s0 == s3) {
                    const float ss = t.step_size[s0];
                    adam_one(p[u].x, m[u].x, v[u].x, g[u].x, ss, t);
                    adam_one(p[u].y, m[u].y, v[u].y, g[u].y, ss, t);
                    adam_one(p[u].z, m[u].z, v[u].z, g[u].z, ss, t);
                    adam_one(p[u].w, m[u].w, v[u].w, g[u].w, ss, t);
                } else {
                    adam_one(p[u].x, m[u].x, v[u].x, g[u].x, t.step_size[segment_of(t, e)], t);
                    adam_one(p[u].y, m[u].y, v[u].y, g[u].y, t.step_size[segment_of(t, e + 1)], t);
                    adam_one(p[u].z, m[u].z, v[u].z, g[u].z, t.step_size[segment_of(t, e + 2)], t);
                    adam_one(p[u].w, m[u].w, v[u].w, g[u].w, t.step_size[segment_of(t, e + 3)], t);
                }
                __stcs(p4 + c, p[u]);
                __stcs(m4 + c, m[u]);
                __stcs(v4 + c, v[u]);
            }
        }
        // The last n % 4 elements.
        const int64_t e = 4 * chunks + tid;
        if (e < n) adam_one(params[e], exp_avg[e], exp_avg_sq[e], grads[e], t.step_size[segment_of(t, e)], t);
    } else {
        for (int64_t e = tid; e < n; e += stride)
            adam_one(params[e], exp_avg[e], exp_avg_sq[e], grads[e], t.step_size[segment_of(t, e)], t);
    }
}

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" int hds_adam_step(int64_t n, float* params, float* exp_avg, float* exp_avg_sq, const float* grads,
                             int segments, const int64_t* segment_ends, const float* segment_lrs, float step,
                             float beta1, float beta2, float one_minus_beta1, float one_minus_beta2, float eps,
                             hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0, HDS_ERR_INVALID, "adam_step: negative length %lld", (long long)n);
    HDS_REQUIRE(segments >= 1 && segments <= HDS_ADAM_MAX_SEGMENTS, HDS_ERR_INVALID,
                "adam_step: %d segments (1 to %d supported)", segments, HDS_ADAM_MAX_SEGMENTS);
    HDS_REQUIRE(segment_ends != nullptr && segment_lrs != nullptr, HDS_ERR_INVALID,
                "adam_step: null segment table");
    HDS_REQUIRE(step >= 1.0f, HDS_ERR_INVALID, "adam_step: step %g must count from 1", (double)step);
    AdamTable t{};
    t.segments = segments;
    int64_t prev = 0;
    // Bias corrections as the reference computes them (powf of the step count, in float).
    const float bc1 = 1.0f - powf(beta1, step);
    for (int s = 0; s < segments; s++) {
        HDS_REQUIRE(segment_ends[s] >= prev, HDS_ERR_INVALID, "adam_step: segment ends must not decrease");
        t.end[s] = segment_ends[s];
        t.step_size[s] = segment_lrs[s] / bc1;
        prev = segment_ends[s];
    }
    HDS_REQUIRE(prev == n, HDS_ERR_INVALID, "adam_step: the last segment ends at %lld, not at n = %lld",
                (long long)prev, (long long)n);
    t.bc2_sqrt = sqrtf(1.0f - powf(beta2, step));
    t.beta2 = beta2;
    t.one_minus_beta1 = one_minus_beta1;
    t.one_minus_beta2 = one_minus_beta2;
    t.eps = eps;
    if (n == 0) return HDS_OK;
    const bool vector = ((reinterpret_cast<uintptr_t>(params) | reinterpret_cast<uintptr_t>(exp_avg) |
                          reinterpret_cast<uintptr_t>(exp_avg_sq) | reinterpret_cast<uintptr_t>(grads)) &
                         15u) == 0;
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t work = vector ? (n / 4 + ADAM_UNROLL - 1) / ADAM_UNROLL : n;
    const int64_t wanted = (work + ADAM_THREADS - 1) / ADAM_THREADS;
    const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(wanted, (int64_t)sms * 8));
    adam_flat_kernel<<<blocks, ADAM_THREADS, 0, stream>>>(n, params, exp_avg, exp_avg_sq, grads, t, vector ? 1 : 0);
    HDS_CHECK_LAUNCH("adam_flat_kernel");
    return HDS_OK;
}
