// render_features_bwd.cu -- backward of the feature blend on tcgen05 tensor cores.
//
// Restates features.cu:350-616 of the reference (render_features_backward + host wrapper): each
// pixel walks its tile's list back to front from its last contributor, recovering T by division,
// and produces dL/dfeatures[g, c] = sum_p w[p, g] dL/dout[p, c] (w = alpha * T), and
// dL/dalpha = T (dot - behind) with dot[p, g] = f[g] . dL/dout[p], which drives the opacity, mean
// and conic gradients.  As in the reference, channels are processed in slices and every slice adds
// its share of the geometric gradients (they are linear in the dots).
//
// Blackwell design.  The two contractions run on the tensor cores; only the per-pixel recurrence
// (T, behind) and the geometric partials stay on the FP32 pipes.  A block owns half a 16x16 tile
// (128 pixels = 128 TMEM lanes) and a slice of CK <= 128 channels:
//   * dL/dout of the block, G[p][c], is staged once in shared memory as bf16 hi + lo
//     (x = hi + lo + O(2^-17 x)), in a layout that is at once the K-major A operand of
//     dot = G F^T and the MN-major A operand of dF^T = G^T W;
//   * producer warps 4-7 walk the tile's list back to front in chunks of 32 entries whose
//     opacity-aware box touches the half tile, gather the chunk's feature slices as bf16 hi + lo,
//     and issue dot[p, k] (M = 128 pixels, N = 32, K = CK) as three MMAs
//     (hi.hi + hi.lo + lo.hi: relative error ~2^-16 against the FP32 sum);
//   * pixel warps 0-3 read their 32 dots from TMEM and run only what is serial per pixel: alpha,
//     the recurrence, w = T * alpha (written as the MN-major B operand, bf16 hi + lo) and
//     u = dL/dalpha * G (fp32); then they issue dF^T[c, k] (M = 128 channels, N = 32,
//     K = 128 pixels), again as three MMAs;
//   * the producers turn u into the geometric gradients -- they are linear in the moments
//     sum_p u {1, dx, dy, dx^2, dx dy, dy^2}, one entry per lane, FP32 -- and drain dF^T from TMEM
//     (lane = channel) into coalesced atomics.
// Stages rotate through a three-deep ring, so gathering, walking and both contractions overlap.
// Every mbarrier wait is bounded; a group that sees one run out stops (decided group-uniformly at a
// barrier), records HDS_ERR_DEVICE for hds_device_status, waits for its own MMAs, frees TMEM and
// returns.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "feature_bwd_common.cuh"

namespace hds {
__device__ int g_backward_status = 0;
}  // namespace hds

#include "feature_bwd_cluster.cuh"

namespace hds {

namespace {

using namespace fbwd;
constexpr int STAGES = 4;
constexpr int MAX_CK = 128; // channels per block (the M of the dF MMA)
// Warp roles: pixel warps 0-7, list warp 8, operand warps 9-12, MMA warp 13.
constexpr int PIXEL_WARPS = 8, LIST_WARP = 8, OPERAND_WARP0 = 9, OPERAND_WARPS = 4, MMA_WARP = 13;
constexpr int THREADS = (MMA_WARP + 1) * 32, PIXEL_THREADS = PIXEL_WARPS * 32;
static_assert(LIST_WARP == PIXEL_WARPS && OPERAND_WARP0 == LIST_WARP + 1 &&
                  MMA_WARP == OPERAND_WARP0 + OPERAND_WARPS,
              "warp roles must partition the block");
enum class Role { Pixel, List, Operand, Mma };
__device__ __forceinline__ Role role_of(int warp) {
    return warp < PIXEL_WARPS ? Role::Pixel
           : warp == LIST_WARP ? Role::List
           : warp < OPERAND_WARP0 + OPERAND_WARPS ? Role::Operand
                                                   : Role::Mma;
}
constexpr int PIXEL_BAR = 1, OPERAND_BAR = 2;
constexpr int G_BYTES = PIX * MAX_CK * 2;  // one bf16 copy of G: [c/8][p][c%8]
constexpr int W_BYTES = PIX * KC * 2;      // one bf16 copy of W: [k/8][p][k%8]
// u = dL/dalpha * G per (pixel, entry), fp32 as [k/4][p][k%4]; the quad rows are padded by 16 bytes
// so that 32 lanes reading one pixel's 32 entries hit 32 different banks.
constexpr int U_QUAD_STRIDE = PIX * 16 + 16;
constexpr int U_BYTES = (KC / 4) * U_QUAD_STRIDE;
// TMEM columns: dots at s*32, dF^T at 128 + s*32, and G as the dot's A operand from G_TMEM (lane =
// pixel; hi: CK / 2 columns of channel pairs, then lo).
constexpr uint32_t TMEM_COLS = 512, G_TMEM = 256;

template <int CK>
struct BwdCfg {
    static constexpr int F_BYTES = KC * CK * 2;  // one bf16 copy of a chunk's features: [c/8][k][c%8]
    // A chunk's features are dead once its dot MMA has run and its weights are written only after
    // that, so F and W share one buffer per stage; once the dF MMA has read W, the buffer also
    // holds the dF transpose ([k][c] fp32, KC * CK * 4 bytes).
    static constexpr int FW_BYTES = F_BYTES > W_BYTES ? 2 * F_BYTES : 2 * W_BYTES;
    static_assert(KC * CK * 4 <= FW_BYTES, "dF transpose must fit the stage buffer");
    static constexpr int STAGE_BYTES = FW_BYTES + U_BYTES;
    static constexpr int SMEM = 2 * G_BYTES + STAGES * STAGE_BYTES + 1024;
    static constexpr int F_LBO = (KC / 8) * 128;  // 512: between 8-channel blocks of F
    // dot = G F^T: A = G from TMEM (lane = pixel, K = channels along the columns),
    //              B = F K-major (SBO 128 between entry groups, LBO 512 between channel blocks).
    static constexpr uint32_t IDESC_DOT = tc::idesc_bf16(128, KC, false, false);
    // dF^T = G^T W: A = G MN-major (SBO 2048 between channel blocks, LBO 128 between pixel groups),
    //               B = W MN-major (SBO 2048 between entry blocks, LBO 128 between pixel groups).
    static constexpr uint32_t IDESC_DF = tc::idesc_bf16(128, KC, true, true);
    static_assert(CK == 32 || CK == 64 || CK == 128, "unsupported slice");
};

template <int CK, bool RGB>
__global__ void __launch_bounds__(THREADS, 1) feature_backward_kernel(
    int C, int width, int height, int tiles_x, int origin_y, int slices, int helper_every,
    const int2* __restrict__ ranges,
    const int32_t* __restrict__ values, const float2* __restrict__ means2D, const float4* __restrict__ conic4,
    const float4* __restrict__ color_opacity, const float* __restrict__ features, const float* __restrict__ final_T_in,
    const int32_t* __restrict__ n_contrib, const float* __restrict__ grad_out, float* __restrict__ grad_means2D,
    float* __restrict__ grad_conics, float* __restrict__ grad_features, float* __restrict__ grad_opacities,
    const float* __restrict__ grad_image, const float* __restrict__ background, float* __restrict__ grad_colors) {
    using Cfg = BwdCfg<CK>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ BwdChunk s_list[LIST_SLOTS];
    __shared__ uint64_t s_ready[STAGES], s_dot_full[STAGES], s_walk_done[STAGES], s_df_full[STAGES];
    __shared__ uint64_t s_list_full[LIST_SLOTS], s_list_free[LIST_SLOTS];
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    __shared__ float s_gp[PIX][3];  // dL/dimage of the block's pixels (the RGB terms of slice 0)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int slice = blockIdx.x % slices;
    // With grad_image, the first slice's blocks also carry the RGB backward: its dot is colour . dL/dpixel
    // and its recurrence the same as the features' (backward.cu:7-164), plus the background term.
    const bool rgb = RGB && slice == 0;
    // As the helper of the cluster kernel (helper_every = M > 0), block group j takes half tile
    // j M + M - 1, the half tiles the clusters skip.
    const int half_id = helper_every > 0 ? (int)(blockIdx.x / slices) * helper_every + helper_every - 1
                                         : (int)(blockIdx.x / slices);
    const int tile = half_id >> 1;
    const int c0 = slice * CK;
    const int x0 = (tile % tiles_x) * TILE;
    const int y0 = (tile / tiles_x) * TILE + (half_id & 1) * 8;
    if (y0 >= height) return;  // the lower half of a bottom-row tile can lie wholly outside the image

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t g_hi = tc::smem_addr(smem), g_lo = g_hi + G_BYTES;
    const uint32_t stage0 = g_hi + 2 * G_BYTES;
    // Stage s: F hi, F lo, W hi, W lo.
    auto f_hi = [&](int s) { return stage0 + s * Cfg::STAGE_BYTES; };
    auto w_hi = [&](int s) { return stage0 + s * Cfg::STAGE_BYTES; };
    auto u_base = [&](int s) { return stage0 + s * Cfg::STAGE_BYTES + Cfg::FW_BYTES; };

    if (warp == 0) tc::tmem_alloc(&s_tmem, TMEM_COLS);
    if (tid == 0) {
        for (int s = 0; s < STAGES; s++) {
            tc::mbar_init(&s_ready[s], 1);
            tc::mbar_init(&s_dot_full[s], 1);
            tc::mbar_init(&s_walk_done[s], 1);
            tc::mbar_init(&s_df_full[s], 1);
        }
        for (int l = 0; l < LIST_SLOTS; l++) {
            tc::mbar_init(&s_list_full[l], 1);
            tc::mbar_init(&s_list_free[l], 1);
        }
        tc::fence_mbar_init();
        s_fail = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s_tmem;
    const int2 range = ranges[tile];

    const Role role = role_of(warp);
    if (role == Role::List) {
        // ------------------------------------------------------------------ list warp 8
        // Hit masks: which entries touch each pixel warp's 8 x 2 block (the pixel warps skip the others).
        list_producer<RGB>(lane, x0, y0, origin_y, width, height, range, values, means2D, conic4, color_opacity, n_contrib,
                           s_list, s_list_full, s_list_free, &s_fail, [&](BwdChunk& ch, int filled) {
                               const bool valid = lane < filled;
                               const float2 m = valid ? ch.mean[lane] : make_float2(0.0f, 0.0f);
                               const float2 e = valid ? ch.ext[lane] : make_float2(-1e30f, -1e30f);
#pragma unroll
                               for (int w = 0; w < 8; w++) {
                                   const float bx0 = (float)(x0 + (w & 1) * 8) + 0.5f;
                                   const float by0 = (float)(y0 + origin_y + ((w & 3) >> 1) * 4 + (w >> 2) * 2) + 0.5f;
                                   const unsigned mask = __ballot_sync(
                                       FULL_MASK, valid && box_hits(m, e, bx0, bx0 + 7.0f, by0, by0 + 1.0f));
                                   if (lane == 0) ch.hits[w] = mask;
                               }
                           });
    } else if (role == Role::Operand) {
        // ------------------------------------------------------------------ operand warps 9-12
        const int otid = tid - OPERAND_WARP0 * 32, ow = otid >> 5;
        const int q4 = warp & 3;                                   // TMEM subpartition of this warp
        const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;      // its lanes (channels of dF^T)

        // Stage G (dL/dout of the half tile and slice) as bf16 hi + lo.  Each warp instruction
        // reads 8 pixels x 64 contiguous bytes and writes two 128-byte runs of shared memory.
        // Two rounds of 2 x CK/16 loads, all of a round issued before its first conversion, so that each
        // thread has 2 CK/16 loads of dL/dout in flight (the staging is bound by their latency).
        constexpr int GROUPS = 2;
#pragma unroll 1
        for (int pp0 = 0; pp0 < 4; pp0 += GROUPS) {
            float4 v[GROUPS][CK / 16];
#pragma unroll
            for (int gi = 0; gi < GROUPS; gi++) {
                const int p = (pp0 + gi) * 32 + ow * 8 + (lane >> 2);
                const int2 lp = half_tile_pixel(p);
                const int px = x0 + lp.x, py = y0 + lp.y;
                const bool in = px < width && py < height;
                const float4* src = reinterpret_cast<const float4*>(grad_out + ((size_t)(in ? py : 0) * width +
                                                                                 (in ? px : 0)) * C + c0);
#pragma unroll
                for (int j = 0; j < CK / 16; j++)
                    v[gi][j] = in ? __ldg(src + j * 4 + (lane & 3)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
#pragma unroll
            for (int gi = 0; gi < GROUPS; gi++) {
                const int p = (pp0 + gi) * 32 + ow * 8 + (lane >> 2);
#pragma unroll
                for (int j = 0; j < CK / 16; j++) {
                    const int c4 = j * 4 + (lane & 3);
                    uint32_t h0, l0, h1, l1;
                    split_bf16(v[gi][j].x, v[gi][j].y, h0, l0);
                    split_bf16(v[gi][j].z, v[gi][j].w, h1, l1);
                    const uint32_t off = (c4 >> 1) * 2048 + p * 16 + (c4 & 1) * 8;
                    st_shared_v2(g_hi + off, h0, h1);
                    st_shared_v2(g_lo + off, l0, l1);
                }
            }
        }
        // The dF MMA reads 128 channel rows of G: zero the rows past the slice.
        for (int i = CK * 16 + otid; i < G_BYTES / 16; i += 128) {  // channel blocks CK/8.. are 2048 B each
            st_shared_v4(g_hi + i * 16, 0u, 0u, 0u, 0u);
            st_shared_v4(g_lo + i * 16, 0u, 0u, 0u, 0u);
        }
        // G also goes to TMEM as the dot's A operand (lane = pixel, column = channel pair), so that
        // the dot MMAs read only their B operand from shared memory.  Each warp copies the rows of
        // its lane quadrant: pixel p's 16-byte block of eight channels is four columns.
        tc::group_sync<OPERAND_BAR>();
        {
            const int p = q4 * 32 + lane;
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const uint32_t src = (half ? g_lo : g_hi) + p * 16;
                const uint32_t dst = tmem + ((uint32_t)(q4 * 32) << 16) + G_TMEM + half * (CK / 2);
#pragma unroll
                for (int cb0 = 0; cb0 < CK / 8; cb0 += 4) {
                    uint32_t r[16];
#pragma unroll
                    for (int b = 0; b < 4; b++)
                        asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                                     : "=r"(r[4 * b]), "=r"(r[4 * b + 1]), "=r"(r[4 * b + 2]), "=r"(r[4 * b + 3])
                                     : "r"(src + (cb0 + b) * 2048));
                    tc::tmem_st16(dst + cb0 * 4, r);
                }
            }
            tc::tmem_wait_st();
        }
        tc::fence_before_sync();

        int n_real = -1;  // number of non-empty chunks, known once the empty chunk arrives
        for (int c = 0;; c++) {
            if (n_real >= 0 && c - STAGES >= n_real) break;  // every chunk is drained
            const int s = c % STAGES, slot = c % LIST_SLOTS;
            const bool fresh = n_real < 0;
            int cnt = 0;
            float4 fv[CK / 16];
            if (fresh) {
                bool bad = false;
                if (otid == 0) {
                    bad = *(volatile int*)&s_fail ||
                          !tc::mbar_wait_bounded(&s_list_full[slot], (c / LIST_SLOTS) & 1, WAIT_LIMIT);
                    if (bad) s_fail = 1;
                }
                if (tc::group_sync_count<OPERAND_BAR>(bad) != 0) break;
                cnt = s_list[slot].count;
                // Issue chunk c's feature loads now; they land while chunk c - STAGES is drained.
                const int k = ow * 8 + (lane >> 2);
                const float4* row =
                    reinterpret_cast<const float4*>(features + (size_t)(k < cnt ? s_list[slot].id[k] : 0) * C + c0);
#pragma unroll
                for (int j = 0; j < CK / 16; j++)
                    fv[j] = k < cnt ? __ldg(row + j * 4 + (lane & 3)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
            if (c >= STAGES) {
                // Drain chunk e = c - STAGES (stage s, list slot e % LIST_SLOTS).
                const int e = c - STAGES;
                const BwdChunk& ce = s_list[e % LIST_SLOTS];
                const uint32_t par = (e / STAGES) & 1;
                bool bad = false;
                if (otid == 0) {
                    bad = *(volatile int*)&s_fail || !tc::mbar_wait_bounded(&s_walk_done[s], par, WAIT_LIMIT);
                    if (bad) s_fail = 1;
                }
                if (tc::group_sync_count<OPERAND_BAR>(bad) != 0) break;
                const int ecnt = ce.count;
                // Geometric gradients of entry k = lane over the pixels of pixel warp q4 (an 8 x 4
                // block): with u = dL/dalpha * G they are linear in sum u {1, dx, dy, dx^2, dx dy, dy^2}.
                if (lane < ecnt) {
                    const float2 m = ce.mean[lane];
                    const float4 q = ce.conic[lane];
                    const float bx = (float)(x0 + (q4 & 1) * 8) + 0.5f, by = (float)(y0 + origin_y + (q4 >> 1) * 4) + 0.5f;
                    const uint8_t* ub = smem + (u_base(s) - g_hi) + (lane >> 2) * U_QUAD_STRIDE + (lane & 3) * 4 +
                                        q4 * 32 * 16;
                    float m0 = 0.0f, mx = 0.0f, my = 0.0f, mxx = 0.0f, mxy = 0.0f, myy = 0.0f;
#pragma unroll
                    for (int i = 0; i < 32; i++) {
                        const float u = *reinterpret_cast<const float*>(ub + i * 16);
                        const float dx = __fsub_rn(bx + (float)(i & 7), m.x), dy = __fsub_rn(by + (float)(i >> 3), m.y);
                        const float ux = u * dx, uy = u * dy;
                        m0 += u;
                        mx += ux;
                        my += uy;
                        mxx = fmaf(ux, dx, mxx);
                        mxy = fmaf(ux, dy, mxy);
                        myy = fmaf(uy, dy, myy);
                    }
                    const int g = ce.id[lane];
                    const float o = q.w;
                    const float v[6] = {m0, o * fmaf(q.y, my, q.x * mx), o * fmaf(q.z, my, q.y * mx), -0.5f * o * mxx,
                                        -o * mxy, -0.5f * o * myy};
                    if (v[0] != 0.0f) atomicAdd(grad_opacities + g, v[0]);
                    if (v[1] != 0.0f) atomicAdd(grad_means2D + 2 * g, v[1]);
                    if (v[2] != 0.0f) atomicAdd(grad_means2D + 2 * g + 1, v[2]);
                    if (v[3] != 0.0f) atomicAdd(grad_conics + 3 * g, v[3]);
                    if (v[4] != 0.0f) atomicAdd(grad_conics + 3 * g + 1, v[4]);
                    if (v[5] != 0.0f) atomicAdd(grad_conics + 3 * g + 2, v[5]);
                    if (rgb) {
                        // dL/dcolour of the entry: sum over the warp's pixels of w dL/dpixel, with w read
                        // back from the stage's W operand (bf16 hi + lo) before the dF transpose reuses it.
                        const uint8_t* wb = smem + (w_hi(s) - g_hi) + (lane >> 3) * 2048 + (lane & 7) * 2 + q4 * 32 * 16;
                        float cr = 0.0f, cg = 0.0f, cb = 0.0f;
#pragma unroll 4
                        for (int i = 0; i < 32; i++) {
                            const uint32_t h = *reinterpret_cast<const uint16_t*>(wb + i * 16);
                            const uint32_t l = *reinterpret_cast<const uint16_t*>(wb + W_BYTES + i * 16);
                            const float w = __uint_as_float(h << 16) + __uint_as_float(l << 16);
                            const float* gp = s_gp[q4 * 32 + i];
                            cr = fmaf(w, gp[0], cr);
                            cg = fmaf(w, gp[1], cg);
                            cb = fmaf(w, gp[2], cb);
                        }
                        if (cr != 0.0f) atomicAdd(grad_colors + 3 * g, cr);
                        if (cg != 0.0f) atomicAdd(grad_colors + 3 * g + 1, cg);
                        if (cb != 0.0f) atomicAdd(grad_colors + 3 * g + 2, cb);
                    }
                }
                // dF of the chunk: wait for its MMA, then drain TMEM (lane = channel).
                if (otid == 0) {
                    bad = *(volatile int*)&s_fail || !tc::mbar_wait_bounded(&s_df_full[s], par, WAIT_LIMIT);
                    if (bad) s_fail = 1;
                }
                if (tc::group_sync_count<OPERAND_BAR>(bad) != 0) break;
                tc::fence_after_sync();
                float v[32];
                tc::tmem_ld32(tmem + lane_base + 128 + s * 32, v);
                tc::fence_before_sync();
                // Transpose dF^T (lane = channel) through stage s's feature buffer -- free, its dot MMA
                // has completed -- into rows of the entry, then add them with float4 atomics.
                uint8_t* tr = smem + (f_hi(s) - g_hi);
                const int cl = q4 * 32 + lane;
                if (cl < CK) {
#pragma unroll
                    for (int k = 0; k < KC; k++)
                        if (k < ecnt) *reinterpret_cast<float*>(tr + (k * CK + cl) * 4) = v[k];
                }
                tc::group_sync<OPERAND_BAR>();
                for (int i = otid; i < ecnt * (CK / 4); i += 128) {
                    const int k = i / (CK / 4), c4 = i % (CK / 4);
                    const float4 d = *reinterpret_cast<const float4*>(tr + (k * CK + 4 * c4) * 4);
                    if (d.x != 0.0f || d.y != 0.0f || d.z != 0.0f || d.w != 0.0f)
                        atomicAdd(reinterpret_cast<float4*>(grad_features + (size_t)ce.id[k] * C + c0) + c4, d);
                }
                tc::group_sync<OPERAND_BAR>();
                if (otid == 0) tc::mbar_arrive(&s_list_free[e % LIST_SLOTS]);
            }
            if (!fresh) continue;
            if (cnt > 0) {
                // Chunk c's features as bf16 hi + lo (zeros past cnt).  Stage s is free: the pixels
                // finished chunk c - STAGES, so its dot MMA has completed.
                const int k = ow * 8 + (lane >> 2);
                const uint32_t fh = f_hi(s), fl = fh + Cfg::F_BYTES;
#pragma unroll
                for (int j = 0; j < CK / 16; j++) {
                    const int c4 = j * 4 + (lane & 3);
                    uint32_t h0, l0, h1, l1;
                    split_bf16(fv[j].x, fv[j].y, h0, l0);
                    split_bf16(fv[j].z, fv[j].w, h1, l1);
                    const uint32_t off = (c4 >> 1) * Cfg::F_LBO + k * 16 + (c4 & 1) * 8;
                    st_shared_v2(fh + off, h0, h1);
                    st_shared_v2(fl + off, l0, l1);
                }
            }
            tc::fence_proxy_async();
            tc::fence_before_sync();
            tc::group_sync<OPERAND_BAR>();
            // Chunk c is published: its list, its features, and a stage whose previous chunk is drained.
            if (otid == 0) tc::mbar_arrive(&s_ready[s]);
            if (cnt == 0) n_real = c;
        }
    } else if (role == Role::Mma) {
        // ------------------------------------------------------------------ MMA warp 13 (one lane)
        // Issues every tensor-core instruction, polling two queues: the dot of the next published
        // chunk, and the dF of the oldest chunk whose walk is done.
        if (lane == 0) {
            int cd = 0, cf = 0, n_end = -1;  // next chunk for dot / dF; the empty chunk's index
            uint64_t* last_bar = nullptr;    // the most recent commit and its phase parity
            uint32_t last_par = 0, idle = 0;
            while (n_end < 0 || cf < n_end) {
                if (*(volatile int*)&s_fail) break;
                bool progress = false;
                if (n_end < 0 && tc::mbar_try_wait(&s_ready[cd % STAGES], (cd / STAGES) & 1)) {
                    const int s = cd % STAGES;
                    if (s_list[cd % LIST_SLOTS].count == 0) {
                        n_end = cd;
                    } else {
                        tc::fence_after_sync();
                        const uint32_t fh = f_hi(s), fl = fh + Cfg::F_BYTES;
#pragma unroll
                        for (int ks = 0; ks < CK / 16; ks++) {
                            const uint32_t ah = tmem + G_TMEM + ks * 8, al = ah + CK / 2;  // A = G from TMEM
                            const uint64_t bh = tc::smem_desc(fh + ks * 2 * Cfg::F_LBO, Cfg::F_LBO, 128);
                            const uint64_t bl = tc::smem_desc(fl + ks * 2 * Cfg::F_LBO, Cfg::F_LBO, 128);
                            const uint32_t d = tmem + s * 32;
                            tc::mma_bf16_ta(d, ah, bh, Cfg::IDESC_DOT, ks > 0 ? 1u : 0u);
                            tc::mma_bf16_ta(d, ah, bl, Cfg::IDESC_DOT, 1u);
                            tc::mma_bf16_ta(d, al, bh, Cfg::IDESC_DOT, 1u);
                        }
                        tc::commit(&s_dot_full[s]);
                        last_bar = &s_dot_full[s];
                        last_par = (cd / STAGES) & 1;
                        cd++;
                    }
                    progress = true;
                }
                if (cf < cd && tc::mbar_try_wait(&s_walk_done[cf % STAGES], (cf / STAGES) & 1)) {
                    // dF^T of chunk cf = G^T W (its weights are in the stage's F/W buffer).
                    const int s = cf % STAGES;
                    tc::fence_after_sync();
                    const uint32_t wh = w_hi(s), wl = wh + W_BYTES;
#pragma unroll
                    for (int ks = 0; ks < PIX / 16; ks++) {
                        const uint64_t ah = tc::smem_desc(g_hi + ks * 256, 128, 2048);
                        const uint64_t al = tc::smem_desc(g_lo + ks * 256, 128, 2048);
                        const uint64_t bh = tc::smem_desc(wh + ks * 256, 128, 2048);
                        const uint64_t bl = tc::smem_desc(wl + ks * 256, 128, 2048);
                        const uint32_t d = tmem + 128 + s * 32;
                        tc::mma_bf16(d, ah, bh, Cfg::IDESC_DF, ks > 0 ? 1u : 0u);
                        tc::mma_bf16(d, ah, bl, Cfg::IDESC_DF, 1u);
                        tc::mma_bf16(d, al, bh, Cfg::IDESC_DF, 1u);
                    }
                    tc::commit(&s_df_full[s]);
                    last_bar = &s_df_full[s];
                    last_par = (cf / STAGES) & 1;
                    cf++;
                    progress = true;
                }
                if (progress) {
                    idle = 0;
                } else if (++idle > WAIT_LIMIT) {
                    s_fail = 1;
                    break;
                }
            }
            // tcgen05 operations complete in issue order: the last commit covers every MMA.
            if (last_bar != nullptr && !tc::mbar_wait_bounded(last_bar, last_par, WAIT_LIMIT)) s_fail = 1;
        }
    } else {  // Role::Pixel
        // ------------------------------------------------------------------ pixel warps 0-7
        // Two threads per pixel: warp w covers 16 pixels of TMEM lane quadrant w & 3 (an 8 x 2
        // block); thread t < 16 and its partner t + 16 share pixel t, and each computes the alphas
        // of half of every group of eight entries (part 0: entries 0-3, part 1: entries 4-7).
        const int quad = warp & 3, half16 = warp >> 2, part = lane >> 4;
        const int p = quad * 32 + half16 * 16 + (lane & 15);
        const int2 lp = half_tile_pixel(p);
        const int px = x0 + lp.x, py = y0 + lp.y;
        const bool inside = px < width && py < height;
        const float cx = (float)px + 0.5f, cy = (float)(py + origin_y) + 0.5f;
        const size_t pix = (size_t)py * width + px;
        float T = inside ? final_T_in[pix] : 0.0f;
        const float fT = T;  // final transmittance: the background's weight
        const int last = inside ? n_contrib[pix] : 0;
        float behind = 0.0f, behind_rgb = 0.0f;
        float gpr = 0.0f, gpg = 0.0f, gpb = 0.0f, bgdot = 0.0f;
        if (rgb) {
            if (inside) {
                gpr = grad_image[3 * pix];
                gpg = grad_image[3 * pix + 1];
                gpb = grad_image[3 * pix + 2];
            }
            bgdot = fmaf(background[2], gpb, fmaf(background[1], gpg, background[0] * gpr));
            if (part == 0) {
                s_gp[p][0] = gpr;
                s_gp[p][1] = gpg;
                s_gp[p][2] = gpb;
            }
        }
        const uint32_t lane_base = (uint32_t)(quad * 32 + half16 * 16) << 16;

        for (int c = 0;; c++) {
            const int s = c % STAGES;
            const BwdChunk& ch = s_list[c % LIST_SLOTS];
            const uint32_t par = (c / STAGES) & 1;
            bool bad = false;
            if (tid == 0) {
                bad = *(volatile int*)&s_fail;
                if (!bad && !tc::mbar_wait_bounded(&s_ready[s], par, WAIT_LIMIT)) bad = true;
                if (!bad && ch.count > 0 && !tc::mbar_wait_bounded(&s_dot_full[s], par, WAIT_LIMIT)) bad = true;
                if (bad) s_fail = 1;
            }
            if (tc::group_sync_count<PIXEL_BAR>(bad, PIXEL_THREADS) != 0) break;
            const int cnt = ch.count;
            if (cnt == 0) break;
            tc::fence_after_sync();

            // Groups of eight entries, in a rolled loop so one group body is all the code the walk
            // needs.  The walk is branch-free: an entry that does not contribute gets alpha 0, for
            // which the recurrence is the identity (T / 1, w = 0, behind kept).  Each thread computes
            // alpha, 1 / (1 - alpha) and G for its four entries; the pair swaps them with the dots,
            // and both run the short serial T / behind chain over all eight.  Each thread writes its
            // half of the group's W block (bf16 hi + lo) and its u quad; the geometric partials
            // leave as u = dL/dalpha * G, summed by the operand warps.
            const uint32_t wh = w_hi(s), wl = wh + W_BYTES, ub = u_base(s) + p * 16;
            const unsigned hits_w = ch.hits[warp];  // entries whose box touches this warp's pixels
#pragma unroll 1
            for (int k0 = 0; k0 < cnt; k0 += 8) {
                const int kb = k0 + 4 * part;  // this thread's four entries
                float d_own[4];
                tc::tmem_ld16x2_4(tmem + lane_base + s * 32 + k0, d_own);
                bool hit[4];
#pragma unroll
                for (int i = 0; i < 4; i++) hit[i] = (hits_w >> (kb + i)) & 1u;
                float w_own[4] = {0.0f, 0.0f, 0.0f, 0.0f}, u_own[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if ((hits_w >> k0) & 0xFFu) {  // uniform per warp
                    float a_own[4], r_own[4], g_own[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float4 q = ch.conic[kb + i];
                        const float2 m = ch.mean[kb + i];
                        const PairAlpha pa = pair_alpha(cx, cy, m.x, m.y, q.x, q.y, q.z, q.w);
                        const float alpha = fminf(MAX_ALPHA, pa.raw);
                        const bool ok = hit[i] && inside && ch.pos[kb + i] < last && alpha >= MIN_ALPHA;
                        a_own[i] = ok ? alpha : 0.0f;
                        r_own[i] = ok ? __fdividef(1.0f, 1.0f - alpha) : 1.0f;
                        // A clamped alpha no longer depends on the gaussian: nothing flows past it.
                        g_own[i] = ok && pa.raw <= MAX_ALPHA ? pa.G : 0.0f;
                    }
                    // Entries 0-3 come from part 0, entries 4-7 from part 1.
                    float a8[8], r8[8], d8[8];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float a_p = __shfl_xor_sync(FULL_MASK, a_own[i], 16);
                        const float r_p = __shfl_xor_sync(FULL_MASK, r_own[i], 16);
                        const float d_p = __shfl_xor_sync(FULL_MASK, d_own[i], 16);
                        a8[i] = part ? a_p : a_own[i];
                        a8[i + 4] = part ? a_own[i] : a_p;
                        r8[i] = part ? r_p : r_own[i];
                        r8[i + 4] = part ? r_own[i] : r_p;
                        d8[i] = part ? d_p : d_own[i];
                        d8[i + 4] = part ? d_own[i] : d_p;
                    }
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        T = T * r8[i];
                        float dL_dalpha = T * (d8[i] - behind);
                        if (rgb) {  // uniform per block
                            const float4 col = ch.col[k0 + i];
                            const float drgb = fmaf(col.z, gpb, fmaf(col.y, gpg, col.x * gpr));
                            // The background is seen through T_final, which this entry's alpha scales.
                            dL_dalpha += T * (drgb - behind_rgb) - fT * r8[i] * bgdot;
                            behind_rgb = fmaf(a8[i], drgb, (1.0f - a8[i]) * behind_rgb);
                        }
                        if ((i >> 2) == part) {  // this thread's entry: a select, not a branch
                            w_own[i & 3] = T * a8[i];
                            u_own[i & 3] = dL_dalpha * g_own[i & 3];
                        }
                        behind = fmaf(a8[i], d8[i], (1.0f - a8[i]) * behind);
                    }
                }
                // W block k0/8 as the MN-major B operand: this pixel's 8 weights are one 16-byte run,
                // of which this thread writes its half.
                uint32_t h0, l0, h1, l1;
                split_bf16(w_own[0], w_own[1], h0, l0);
                split_bf16(w_own[2], w_own[3], h1, l1);
                st_shared_v2(wh + (k0 >> 3) * 2048 + p * 16 + part * 8, h0, h1);
                st_shared_v2(wl + (k0 >> 3) * 2048 + p * 16 + part * 8, l0, l1);
                st_shared_v4(ub + ((k0 >> 2) + part) * U_QUAD_STRIDE, __float_as_uint(u_own[0]),
                             __float_as_uint(u_own[1]), __float_as_uint(u_own[2]), __float_as_uint(u_own[3]));
            }
            tc::fence_proxy_async();
            tc::fence_before_sync();
            tc::group_sync<PIXEL_BAR>(PIXEL_THREADS);
            if (tid == 0) tc::mbar_arrive(&s_walk_done[s]);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
    if (tid == 0 && s_fail) atomicExch(&g_backward_status, HDS_ERR_DEVICE);
}

template <int CK>
int launch_backward(int D, int width, int height, int origin_y, const int32_t* tile_ranges, const int32_t* values,
                    const float* means2D, const float* conic4, const float* color_opacity, const float* features,
                    const float* final_T, const int32_t* n_contrib, const float* grad_output, float* grad_features,
                    float* grad_means2D, float* grad_conics, float* grad_opacities, const float* grad_image,
                    const float* background, float* grad_colors, cudaStream_t stream, int helper_every = 0) {
    using Cfg = BwdCfg<CK>;
    auto kernel = grad_image != nullptr ? feature_backward_kernel<CK, true> : feature_backward_kernel<CK, false>;
    HDS_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    const int tx = tiles_for(width), ty = tiles_for(height), slices = D / CK;
    const int halves = 2 * tx * ty;
    const int groups = helper_every > 0 ? halves / helper_every : halves;
    if (groups == 0) return HDS_OK;
    kernel<<<groups * slices, THREADS, Cfg::SMEM, stream>>>(
        D, width, height, tx, origin_y, slices, helper_every, reinterpret_cast<const int2*>(tile_ranges), values,
        reinterpret_cast<const float2*>(means2D), reinterpret_cast<const float4*>(conic4),
        reinterpret_cast<const float4*>(color_opacity), features, final_T, n_contrib, grad_output, grad_means2D,
        grad_conics, grad_features, grad_opacities, grad_image, background, grad_colors);
    HDS_CHECK_LAUNCH("feature_backward_kernel");
    return HDS_OK;
}

}  // namespace

namespace {

// Whether D channels run on the four-block clusters: by default at 512 channels, where they are the
// faster kernel (the RGB backward rides in their walk); HDS_FEATURE_BWD_CLUSTER=1 also selects them at
// 256 channels and =0 never.  Read per call, so a process can switch.
bool cluster_backward_enabled(int D) {
    const char* v = getenv("HDS_FEATURE_BWD_CLUSTER");
    if (v != nullptr && strcmp(v, "0") == 0) return false;
    if (v != nullptr && strcmp(v, "1") == 0) return D >= 256;
    return D == 512;
}

// The four-block clusters of the 512-channel backward fit 33 at a time on a B200 (132 SMs): its
// GPCs do not all hold a multiple of four SMs.  A helper launch of the one-block kernel on a second
// stream takes every M-th half tile; its single-SM blocks run on the SMs no cluster can use, and
// after the clusters drain, on all of them.  HDS_FEATURE_BWD_HELPER: unset = every 14th half tile
// (on the 1.18M-gaussian bench view the backward takes 7.42 ms without a helper and 7.26, 7.19 and
// 7.16 ms with M = 6, 10 and 14), "0" = no helper, an integer M >= 2 = every M-th.  Read per call.
int helper_every() {
    const char* v = getenv("HDS_FEATURE_BWD_HELPER");
    if (v == nullptr || *v == '\0') return 14;
    const int m = atoi(v);
    return m >= 2 ? m : 0;
}

// The helper's stream and its fork / join events, one set per device, created on first use and kept
// for the life of the process.  The stream does not synchronise with the legacy default stream, so
// only the events order it.  The mutex keeps each call's fork, launches and join together.
constexpr int kMaxDevices = 64;
struct HelperStream {
    cudaStream_t stream = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
std::mutex g_helper_mutex;
HelperStream g_helper[kMaxDevices];

template <class ClusterLaunch, class HelperLaunch>
int launch_with_helper(cudaStream_t stream, ClusterLaunch&& clusters, HelperLaunch&& helper) {
    int dev = -1;
    HDS_CHECK_CUDA(cudaGetDevice(&dev));
    HDS_REQUIRE(dev >= 0 && dev < kMaxDevices, HDS_ERR_INVALID, "feature backward: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_helper_mutex);
    HelperStream& h = g_helper[dev];
    if (h.stream == nullptr) {
        HDS_CHECK_CUDA(cudaStreamCreateWithFlags(&h.stream, cudaStreamNonBlocking));
        HDS_CHECK_CUDA(cudaEventCreateWithFlags(&h.fork, cudaEventDisableTiming));
        HDS_CHECK_CUDA(cudaEventCreateWithFlags(&h.join, cudaEventDisableTiming));
    }
    HDS_CHECK_CUDA(cudaEventRecord(h.fork, stream));
    if (int rc = clusters(stream)) return rc;  // launched first: its clusters take the SMs they can
    HDS_CHECK_CUDA(cudaStreamWaitEvent(h.stream, h.fork, 0));
    if (int rc = helper(h.stream)) return rc;
    HDS_CHECK_CUDA(cudaEventRecord(h.join, h.stream));
    HDS_CHECK_CUDA(cudaStreamWaitEvent(stream, h.join, 0));
    return HDS_OK;
}

// grad_image (with background and grad_colors) adds the RGB backward to the same walk; NULL leaves
// it out (the reference's rasterize_features_backward).
int features_backward(int n, int channels, int slice_width, int width, int height, int origin_y,
                      const float* grad_output,
                      const float* features, const float* means2D, const float* conic4, const float* color_opacity,
                      const int32_t* values_sorted, const int32_t* tile_ranges, const float* final_T,
                      const int32_t* n_contrib, float* grad_features, float* grad_means2D, float* grad_conics,
                      float* grad_opacities, bool accumulate_features, const float* grad_image,
                      const float* background, float* grad_colors, void* workspace, size_t workspace_bytes,
                      cudaStream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0, HDS_ERR_INVALID, "rasterize_features_backward: bad sizes");
    HDS_REQUIRE(origin_y >= 0 && origin_y % TILE == 0, HDS_ERR_INVALID,
                "rasterize_features_backward: origin_y %d must be a non-negative multiple of 16", origin_y);
    HDS_REQUIRE((int64_t)channels * width * height <= INT32_MAX, HDS_ERR_TOO_LARGE,
                "a %dx%d image of %d channels overflows the feature kernels' int indices", width, height, channels);
    // The (channels, slice) pairs the reference dispatches (features.cu:601-612).
    const int D = channels, Wd = slice_width;
    const bool supported = (D == 32 && Wd == 32) || (D == 64 && (Wd == 64 || Wd == 32)) ||
                           (D == 128 && (Wd == 128 || Wd == 64 || Wd == 32)) || (D == 256 && (Wd == 128 || Wd == 64)) ||
                           (D == 512 && (Wd == 128 || Wd == 64));
    HDS_REQUIRE(supported, HDS_ERR_UNSUPPORTED, "no feature backward for %d channels in slices of %d", D, Wd);
    HDS_REQUIRE(((uintptr_t)features & 15) == 0 && ((uintptr_t)grad_output & 15) == 0 &&
                    ((uintptr_t)grad_features & 15) == 0,
                HDS_ERR_INVALID, "rasterize_features_backward: features, grad_output and grad_features must be 16-byte aligned");
    HDS_REQUIRE(grad_image == nullptr || (background != nullptr && grad_colors != nullptr), HDS_ERR_INVALID,
                "rasterize_backward_fused: grad_image needs background and grad_colors");
    HDS_REQUIRE(((uintptr_t)workspace & 255) == 0, HDS_ERR_INVALID,
                "rasterize_backward_fused: the workspace must be 256-byte aligned");
    if (n == 0) return HDS_OK;
    if (!accumulate_features) HDS_CHECK_CUDA(cudaMemsetAsync(grad_features, 0, sizeof(float) * (size_t)n * D, stream));
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_means2D, 0, sizeof(float) * 2 * (size_t)n, stream));
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_conics, 0, sizeof(float) * 3 * (size_t)n, stream));
    HDS_CHECK_CUDA(cudaMemsetAsync(grad_opacities, 0, sizeof(float) * (size_t)n, stream));
    if (grad_image != nullptr) HDS_CHECK_CUDA(cudaMemsetAsync(grad_colors, 0, sizeof(float) * 3 * (size_t)n, stream));
    // The slice width only selects the reference's kernel instantiation; the sums are the same for
    // any slicing.  One block per half tile and slice of min(D, 128) channels (one walk per slice), or
    // four-block clusters (slices of D / 4, one walk per pixel).
    if (cluster_backward_enabled(D)) {
        // With a workspace the half tiles' lists are cut by one kernel ahead of the clusters.
        const HalfTileLists lists = half_tile_lists_in(workspace, workspace_bytes, tiles_for(width) * tiles_for(height));
        const HalfTileLists* packed = lists.capacity > 0 ? &lists : nullptr;
        const int m = helper_every();
        if (D == 512 && m > 0 && (2 * tiles_for(width) * tiles_for(height)) / m > 0) {
            return launch_with_helper(
                stream,
                [&](cudaStream_t st) {
                    return clus::launch_backward_cluster<128>(D, width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, final_T, n_contrib, grad_output, grad_features, grad_means2D, grad_conics, grad_opacities, grad_image, background, grad_colors, st, m, packed);
                },
                [&](cudaStream_t st) {
                    return launch_backward<128>(D, width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, final_T, n_contrib, grad_output, grad_features, grad_means2D, grad_conics, grad_opacities, grad_image, background, grad_colors, st, m);
                });
        }
        if (D == 256)
            return clus::launch_backward_cluster<64>(D, width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, final_T, n_contrib, grad_output, grad_features, grad_means2D, grad_conics, grad_opacities, grad_image, background, grad_colors, stream, 0, packed);
        return clus::launch_backward_cluster<128>(D, width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, final_T, n_contrib, grad_output, grad_features, grad_means2D, grad_conics, grad_opacities, grad_image, background, grad_colors, stream, 0, packed);
    }
    switch (D) {
        case 32: return launch_backward<32>(D, width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, final_T, n_contrib, grad_output, grad_features, grad_means2D, grad_conics, grad_opacities, grad_image, background, grad_colors, stream);
        case 64: return launch_backward<64>(D, width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, final_T, n_contrib, grad_output, grad_features, grad_means2D, grad_conics, grad_opacities, grad_image, background, grad_colors, stream);
        default: return launch_backward<128>(D, width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, final_T, n_contrib, grad_output, grad_features, grad_means2D, grad_conics, grad_opacities, grad_image, background, grad_colors, stream);
    }
}

}  // namespace

int read_and_clear_backward_status(int* status, cudaStream_t stream) {
    int zero = 0;
    HDS_CHECK_CUDA(cudaMemcpyFromSymbolAsync(status, g_backward_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream));
    HDS_CHECK_CUDA(cudaMemcpyToSymbolAsync(g_backward_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream));
    return HDS_OK;
}

}  // namespace hds

using namespace hds;

extern "C" int hds_render_features_backward(int n, int channels, int slice_width, int width, int height,
                                            int origin_y, const float* grad_output, const float* features, const float* means2D,
                                            const float* conic4, const float* color_opacity,
                                            const int32_t* values_sorted, const int32_t* tile_ranges,
                                            const float* final_T, const int32_t* n_contrib, float* grad_features,
                                            float* grad_means2D, float* grad_conics, float* grad_opacities,
                                            hds_stream_t stream) {
    return features_backward(n, channels, slice_width, width, height, origin_y, grad_output, features, means2D, conic4,
                             color_opacity, values_sorted, tile_ranges, final_T, n_contrib, grad_features,
                             grad_means2D, grad_conics, grad_opacities, false, nullptr, nullptr, nullptr, nullptr, 0, stream);
}

extern "C" int hds_render_features_backward_accumulate(int n, int channels, int slice_width, int width, int height,
                                                       int origin_y, const float* grad_output, const float* features,
                                                       const float* means2D, const float* conic4,
                                                       const float* color_opacity, const int32_t* values_sorted,
                                                       const int32_t* tile_ranges, const float* final_T,
                                                       const int32_t* n_contrib, float* grad_features,
                                                       float* grad_means2D, float* grad_conics, float* grad_opacities,
                                                       hds_stream_t stream) {
    return features_backward(n, channels, slice_width, width, height, origin_y, grad_output, features, means2D, conic4,
                             color_opacity, values_sorted, tile_ranges, final_T, n_contrib, grad_features,
                             grad_means2D, grad_conics, grad_opacities, true, nullptr, nullptr, nullptr, nullptr, 0, stream);
}

extern "C" int hds_render_backward_fused(int n, int channels, int width, int height, int origin_y,
                                         const float* grad_image,
                                         const float* background, const float* grad_feature_image,
                                         const float* features, const float* means2D, const float* conic4,
                                         const float* color_opacity, const int32_t* values_sorted,
                                         const int32_t* tile_ranges, const float* final_T, const int32_t* n_contrib,
                                         float* grad_colors, float* grad_features, float* grad_means2D,
                                         float* grad_conics, float* grad_opacities, int accumulate_features,
                                         void* workspace, size_t workspace_bytes, hds_stream_t stream) {
    return features_backward(n, channels, channels < 128 ? channels : 128, width, height, origin_y,
                             grad_feature_image, features,
                             means2D, conic4, color_opacity, values_sorted, tile_ranges, final_T, n_contrib,
                             grad_features, grad_means2D, grad_conics, grad_opacities, accumulate_features != 0,
                             grad_image, background, grad_colors, workspace, workspace_bytes, stream);
}

extern "C" size_t hds_backward_workspace_bytes(int64_t pairs, int width, int height) {
    if (pairs < 0 || width <= 0 || height <= 0) return 0;
    return half_tile_lists_bytes(pairs, tiles_for(width) * tiles_for(height));
}
