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
// Layout and traffic: one 32-byte load of each of the four streams per thread and iteration (the
// 256-bit ld.global.v8 of sm_100, no L1 allocation: each byte is touched once), grid-stride over
// groups of eight elements.  Measured on the B200 over 675M elements, this form moves 28 B/element at
// about 0.9 of the copy bandwidth, while four 16-byte chunks in flight per thread reach only 0.6: the
// additional loads in flight slow the DRAM down instead of hiding its latency.  A group that straddles
// two segments, or the tail of a length that is not a multiple of eight, goes element by element;
// buffers that are not 32-byte aligned take the element path throughout.
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
constexpr int ADAM_VEC = 8;  // elements per 32-byte vector

struct Vec8 {
    float x[ADAM_VEC];
};

__device__ __forceinline__ Vec8 ld_vec8(const float* p) {
    Vec8 r;
    asm volatile("ld.global.L1::no_allocate.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=f"(r.x[0]), "=f"(r.x[1]), "=f"(r.x[2]), "=f"(r.x[3]), "=f"(r.x[4]), "=f"(r.x[5]), "=f"(r.x[6]),
                   "=f"(r.x[7])
                 : "l"(p));
    return r;
}

__device__ __forceinline__ void st_vec8(float* p, const Vec8& r) {
    asm volatile("st.global.L1::no_allocate.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "f"(r.x[0]),
                 "f"(r.x[1]), "f"(r.x[2]), "f"(r.x[3]), "f"(r.x[4]), "f"(r.x[5]), "f"(r.x[6]), "f"(r.x[7])
                 : "memory");
}

__global__ void __launch_bounds__(ADAM_THREADS) adam_flat_kernel(int64_t n, float* __restrict__ params,
                                                                 float* __restrict__ exp_avg,
                                                                 float* __restrict__ exp_avg_sq,
                                                                 const float* __restrict__ grads, AdamTable t,
                                                                 int vector) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vector) {
        const int64_t groups = n / ADAM_VEC;
        for (int64_t c = tid; c < groups; c += stride) {
            const int64_t e = c * ADAM_VEC;
            Vec8 p = ld_vec8(params + e), m = ld_vec8(exp_avg + e), v = ld_vec8(exp_avg_sq + e);
            const Vec8 g = ld_vec8(grads + e);
            const int s0 = segment_of(t, e), s7 = segment_of(t, e + ADAM_VEC - 1);
            if (s0 == s7) {
                const float ss = t.step_size[s0];
#pragma unroll
                for (int i = 0; i < ADAM_VEC; i++) adam_one(p.x[i], m.x[i], v.x[i], g.x[i], ss, t);
            } else {
#pragma unroll
                for (int i = 0; i < ADAM_VEC; i++)
                    adam_one(p.x[i], m.x[i], v.x[i], g.x[i], t.step_size[segment_of(t, e + i)], t);
            }
            st_vec8(params + e, p);
            st_vec8(exp_avg + e, m);
            st_vec8(exp_avg_sq + e, v);
        }
        // The last n % 8 elements.
        const int64_t e = groups * ADAM_VEC + tid;
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
                         31u) == 0;
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int64_t work = vector ? n / ADAM_VEC + 1 : n;
    const int64_t wanted = (work + ADAM_THREADS - 1) / ADAM_THREADS;
    const unsigned blocks = (unsigned)std::max<int64_t>(1, std::min<int64_t>(wanted, (int64_t)sms * 8));
    adam_flat_kernel<<<blocks, ADAM_THREADS, 0, stream>>>(n, params, exp_avg, exp_avg_sq, grads, t, vector ? 1 : 0);
    HDS_CHECK_LAUNCH("adam_flat_kernel");
    return HDS_OK;
}
