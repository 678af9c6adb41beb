// feature_bwd_cluster.cuh -- the feature backward for 256 and 512 channels: one four-block cluster
// per half tile, so that the per-pixel walk runs once per pixel instead of once per channel slice.
//
// The backward of features.cu:350-616 splits into a part that is per channel slice -- the dot
// dot[p, k] = f[k] . dL/dout[p] and dL/dfeatures -- and a part that is per pixel and needs the whole
// dot: the transmittance walk (alpha, T, w = alpha T, dL/dalpha) and the geometric gradients.
// Block r of the cluster owns channel slice r (CK = C / 4 channels) and pixel quadrant r (32 of the
// half tile's 128 pixels, TMEM lanes 32r..32r+31):
//   * each block computes its slice's dot for all 128 pixels on the tensor cores (split bf16, as the
//     one-block kernel), and its drain warp q sends quadrant q of it to block q over distributed
//     shared memory as soon as it is in TMEM, chunks ahead of the walk;
//   * block r adds the four partial dots of its quadrant and walks its 32 pixels with eight
//     threads per pixel: each thread takes four consecutive entries of the 32-entry chunk, the
//     eight segments are joined by a scan of their affine maps (T_out = P T_in,
//     behind_out = A behind_in + B), and then each thread runs its own four steps;
//   * block r writes its quadrant of W = alpha T (bf16 hi + lo) into all four blocks, which then
//     compute their slice's dF^T = G^T W on the tensor cores and add it to dL/dfeatures;
//   * block r's operand warps reduce u = dL/dalpha G over its quadrant into the geometric
//     gradients, and with grad_image the walk also carries the RGB backward (backward.cu:7-164)
//     for the block's pixels;
//   * block r's drain warps also move each chunk's dF out of TMEM and add it into dL/dfeatures
//     (one coalesced reduction per entry and warp), concurrently with the operand warps' geometry
//     and feature staging.
// The exchanges are asynchronous stores into the peer's shared memory (st.async) that complete bytes
// of the peer's mbarrier: the sender never waits, and the receiver's barrier phase completes once its
// local writers have arrived (one of them posting the bytes the three peers owe) and every byte has
// landed.  Buffer reuse needs no extra barrier: a block sends chunk c's partial only after its dot
// MMA of chunk c, which follows its dF MMA of chunk c - STAGES, which needed every owner's W of chunk
// c - STAGES -- sent after that owner finished reading its receive buffer.  Every wait is bounded; on
// a timeout a block records HDS_ERR_DEVICE, and its peers time out in turn.  A block whose phases all
// completed has received every byte addressed to it; a block that timed out waits after the final
// cluster barrier for stores still in flight before its shared memory is released.
#pragma once

#include "feature_bwd_common.cuh"

namespace hds {
namespace {
namespace clus {

using namespace fbwd;
constexpr int CLUSTER = 4;           // blocks per half tile: channel slices, and the walk's pixel quadrants
constexpr int QPIX = PIX / CLUSTER;  // 32 pixels per quadrant
constexpr int STAGES = 4;
// Warp roles: pixel warps 0-7, list warp 8, operand warps 9-12, MMA warp 13, drain warps 14-17.
constexpr int PIXEL_WARPS = 8, LIST_WARP = 8, OPERAND_WARP0 = 9, OPERAND_WARPS = 4, MMA_WARP = 13;
constexpr int DRAIN_WARP0 = 14, DRAIN_WARPS = 4;
constexpr int THREADS = (DRAIN_WARP0 + DRAIN_WARPS) * 32;
static_assert(LIST_WARP == PIXEL_WARPS && OPERAND_WARP0 == LIST_WARP + 1 &&
                  MMA_WARP == OPERAND_WARP0 + OPERAND_WARPS && DRAIN_WARP0 == MMA_WARP + 1,
              "warp roles must partition the block");
static_assert(PIXEL_WARPS * 32 == QPIX * 8, "eight walk threads per pixel of the quadrant");
static_assert(OPERAND_WARPS == 4 && DRAIN_WARPS == 4, "four consecutive warps reach all four TMEM lane quadrants");
enum class Role { Pixel, List, Operand, Mma, Drain };
__device__ __forceinline__ Role role_of(int warp) {
    return warp < PIXEL_WARPS ? Role::Pixel
           : warp == LIST_WARP ? Role::List
           : warp < OPERAND_WARP0 + OPERAND_WARPS ? Role::Operand
           : warp == MMA_WARP ? Role::Mma
                              : Role::Drain;
}
constexpr int OPERAND_BAR = 2, DRAIN_BAR = 3;
// Polls without progress before a multi-queue polling loop (MMA warp, drain warps) gives up: their
// test_wait never suspends, so a poll costs tens of cycles, not try_wait's bounded suspension.
constexpr uint32_t POLL_LIMIT = 1u << 26;
constexpr int G_BYTES = PIX * 128 * 2;  // one bf16 copy of G: [c/8][p][c%8], 128 channel rows (the dF M)
// One bf16 copy of W as [p/8][k/8][p%8][k%8], so that quadrant q is the 2 KB at 2048 q.
constexpr int W_BYTES = PIX * KC * 2;
constexpr int W_QUAD_BYTES = W_BYTES / CLUSTER;
// The owner's partial dots: [slice][pixel][entry] fp32, the 16-byte groups of a pixel row permuted
// by (pixel % 8) so that both the senders' and the walk's 16-byte accesses are conflict-free.
constexpr int RECV_SLICE_BYTES = QPIX * KC * 4;
constexpr int RECV_BYTES = CLUSTER * RECV_SLICE_BYTES;
// u = dL/dalpha G of the quadrant: [pixel][entry] fp32, 16-byte groups permuted by 2 (pixel / 8).
constexpr int U_BYTES = QPIX * KC * 4;
// TMEM columns: dots at s*32, dF^T at 128 + s*32, G as the dot's A operand from G_TMEM (lane =
// pixel; hi: CK / 2 columns of channel pairs, then lo), and G^T as the dF's A operand from GT_TMEM
// (lane = channel, rows past the slice zero; hi: 64 columns of pixel pairs, then lo).
constexpr uint32_t TMEM_COLS = 512, G_TMEM = 256, GT_TMEM = 384;

template <int CK>
struct Cfg {
    static constexpr int F_BYTES = KC * CK * 2;  // one bf16 copy of a chunk's features: [c/8][k][c%8]
    // F, then W (from all four blocks), then the dF transpose share one buffer per stage.
    static constexpr int FW_BYTES = (2 * F_BYTES > 2 * W_BYTES ? 2 * F_BYTES : 2 * W_BYTES);
    static_assert(KC * CK * 4 <= FW_BYTES, "dF transpose must fit the stage buffer");
    static constexpr int STAGE_BYTES = FW_BYTES + RECV_BYTES + U_BYTES;
    static constexpr int SMEM = 2 * G_BYTES + STAGES * STAGE_BYTES + 1024;
    static constexpr int F_LBO = (KC / 8) * 128;
    static constexpr uint32_t IDESC_DOT = tc::idesc_bf16(128, KC, false, false);
    static constexpr uint32_t IDESC_DF = tc::idesc_bf16(128, KC, false, true);  // A = G^T from TMEM
    static_assert(CK == 64 || CK == 128, "cluster slices are 64 or 128 channels");
};

// Byte offset of W element (pixel p, entry k) within one bf16 copy.
__device__ __forceinline__ uint32_t w_offset(int p, int k) {
    return (uint32_t)((p >> 3) * 512 + (k >> 3) * 128 + (p & 7) * 16 + (k & 7) * 2);
}

__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ float4 ld_shared_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

// PACKED: the half tiles' lists were cut ahead (cut_half_tile_lists_kernel, `lists`); otherwise each
// block's list warp cuts them from the tile lists.
template <int CK, bool RGB, bool PACKED>
__global__ void __cluster_dims__(CLUSTER, 1, 1) __launch_bounds__(THREADS, 1) feature_backward_cluster_kernel(
    int C, int width, int height, int tiles_x, int origin_y, int helper_every, const int2* __restrict__ ranges,
    const int32_t* __restrict__ values,
    const float2* __restrict__ means2D, const float4* __restrict__ conic4, const float4* __restrict__ color_opacity,
    const float* __restrict__ features, const float* __restrict__ final_T_in, const int32_t* __restrict__ n_contrib,
    const float* __restrict__ grad_out, float* __restrict__ grad_means2D, float* __restrict__ grad_conics,
    float* __restrict__ grad_features, float* __restrict__ grad_opacities, const float* __restrict__ grad_image,
    const float* __restrict__ background, float* __restrict__ grad_colors, HalfTileLists lists) {
    using K = Cfg<CK>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ BwdChunk s_list[LIST_SLOTS];
    __shared__ uint64_t s_ready[STAGES], s_dot_full[STAGES], s_recv_full[STAGES], s_w_full[STAGES];
    __shared__ uint64_t s_walk_done[STAGES], s_df_full[STAGES], s_tmem_free[STAGES];
    __shared__ uint64_t s_list_full[LIST_SLOTS], s_list_free[LIST_SLOTS];
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail;
    __shared__ float s_gp[QPIX][3];  // dL/dimage of the quadrant's pixels (RGB)

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank = (int)tc::cluster_rank();
    // With a helper kernel taking every helper_every-th half tile (M > 1), cluster c takes the c-th of
    // the others: half tiles j M .. j M + M - 2 for j = c / (M - 1).
    const int cidx = blockIdx.x / CLUSTER;
    const int half_id = helper_every > 1 ? (cidx / (helper_every - 1)) * helper_every + cidx % (helper_every - 1) : cidx;
    const int tile = half_id >> 1;
    const int c0 = rank * CK;
    const int x0 = (tile % tiles_x) * TILE;
    const int y0 = (tile / tiles_x) * TILE + (half_id & 1) * 8;
    if (y0 >= height) return;  // the lower half of a bottom-row tile: the whole cluster leaves

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t g_hi = tc::smem_addr(smem), g_lo = g_hi + G_BYTES;
    const uint32_t stage0 = g_hi + 2 * G_BYTES;
    auto fw = [&](int s) { return stage0 + s * K::STAGE_BYTES; };  // F hi, F lo | W hi, W lo | dF^T
    auto recv = [&](int s) { return stage0 + s * K::STAGE_BYTES + K::FW_BYTES; };
    auto ubuf = [&](int s) { return stage0 + s * K::STAGE_BYTES + K::FW_BYTES + RECV_BYTES; };

    if (warp == 0) tc::tmem_alloc(&s_tmem, TMEM_COLS);
    if (tid == 0) {
        for (int s = 0; s < STAGES; s++) {
            tc::mbar_init(&s_ready[s], 1);
            tc::mbar_init(&s_dot_full[s], 1);
            tc::mbar_init(&s_recv_full[s], 1);            // the drain warp storing this block's own quadrant
            tc::mbar_init(&s_w_full[s], PIXEL_WARPS);     // the pixel warps writing this block's quadrant
            tc::mbar_init(&s_walk_done[s], PIXEL_WARPS);
            tc::mbar_init(&s_df_full[s], 1);
            tc::mbar_init(&s_tmem_free[s], DRAIN_WARPS);  // every drain warp has read the chunk's dF
        }
        for (int l = 0; l < LIST_SLOTS; l++) {
            tc::mbar_init(&s_list_full[l], 1);
            // A chunk's entries are read last by the operand warps (geometry) and the drain warps.
            tc::mbar_init(&s_list_free[l], OPERAND_WARPS + DRAIN_WARPS);
        }
        tc::fence_mbar_init();
        s_fail = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::cluster_sync();  // every block's barriers exist before a peer arrives on them
    tc::fence_after_sync();
    const uint32_t tmem = s_tmem;
    const int2 range = ranges[tile];

    const Role role = role_of(warp);
    if (role == Role::List) {
        // ------------------------------------------------------------------ list warp 8
        // Every block of the cluster takes the same chunks (same half tile, same inputs); the hit
        // mask is its own quadrant's (an 8 x 4 block).
        auto mark_hits = [&](BwdChunk& ch, int filled) {
            const bool valid = lane < filled;
            const float2 m = valid ? ch.mean[lane] : make_float2(0.0f, 0.0f);
            const float2 e = valid ? ch.ext[lane] : make_float2(-1e30f, -1e30f);
            const float bx0 = (float)(x0 + (rank & 1) * 8) + 0.5f;
            const float by0 = (float)(y0 + origin_y + (rank >> 1) * 4) + 0.5f;
            const unsigned mask =
                __ballot_sync(FULL_MASK, valid && box_hits(m, e, bx0, bx0 + 7.0f, by0, by0 + 3.0f));
            if (lane == 0) ch.hits[0] = mask;
        };
        if (PACKED)
            list_reader<RGB>(lane, half_id, range, lists, s_list, s_list_full, s_list_free, &s_fail, mark_hits);
        else
            list_producer<RGB>(lane, x0, y0, origin_y, width, height, range, values, means2D, conic4, color_opacity,
                               n_contrib, s_list, s_list_full, s_list_free, &s_fail, mark_hits);
    } else if (role == Role::Operand) {
        // ------------------------------------------------------------------ operand warps 9-12
        const int otid = tid - OPERAND_WARP0 * 32, ow = otid >> 5;
        const int q4 = warp & 3;  // TMEM subpartition of this warp

        // Stage G (dL/dout of the half tile and this block's slice) as bf16 hi + lo.
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
        for (int i = CK * 16 + otid; i < G_BYTES / 16; i += 128) {
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
            // And G^T as the dF MMA's A operand: lane = channel c (this warp's 32), column j = pixels
            // 2j and 2j + 1; the staged rows past the slice are zero.
            const int c = q4 * 32 + lane;
#pragma unroll
            for (int half = 0; half < 2; half++) {
                const uint32_t src = (half ? g_lo : g_hi) + (c >> 3) * 2048 + (c & 7) * 2;
                const uint32_t dst = tmem + ((uint32_t)(q4 * 32) << 16) + GT_TMEM + half * (PIX / 2);
#pragma unroll 1
                for (int j0 = 0; j0 < PIX / 2; j0 += 16) {
                    uint32_t r[16];
#pragma unroll
                    for (int t = 0; t < 16; t++) {
                        const uint32_t a = src + (uint32_t)(2 * (j0 + t)) * 16;
                        uint16_t lo16, hi16;
                        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(lo16) : "r"(a));
                        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(hi16) : "r"(a + 16));
                        r[t] = (uint32_t)lo16 | ((uint32_t)hi16 << 16);
                    }
                    tc::tmem_st16(dst + j0, r);
                }
            }
            tc::tmem_wait_st();
        }
        tc::fence_before_sync();

        int n_real = -1;  // number of non-empty chunks, known once the empty chunk arrives
        for (int c = 0;; c++) {
            if (n_real >= 0 && c - STAGES >= n_real) break;  // every chunk's geometry is reduced
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
                // Issue chunk c's feature loads now; they land while chunk c - STAGES's geometry is reduced.
                const int k = ow * 8 + (lane >> 2);
                const float4* row =
                    reinterpret_cast<const float4*>(features + (size_t)(k < cnt ? s_list[slot].id[k] : 0) * C + c0);
#pragma unroll
                for (int j = 0; j < CK / 16; j++)
                    fv[j] = k < cnt ? __ldg(row + j * 4 + (lane & 3)) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
            if (c >= STAGES) {
                // Geometric gradients of chunk e = c - STAGES (stage s, list slot e % LIST_SLOTS).
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
                {
                    // Geometric gradients over the quadrant: lane = (pixel row g, entry k); with
                    // u = dL/dalpha G they are linear in sum u {1, dx, dy, dx^2, dx dy, dy^2}, and dy
                    // is constant along a row.  The four rows are then added across lanes.
                    const int k = ow * 8 + (lane & 7), g = lane >> 3;
                    const bool kv = k < ecnt;
                    const float2 m = kv ? ce.mean[k] : make_float2(0.0f, 0.0f);
                    const float bx = (float)(x0 + (rank & 1) * 8) + 0.5f;
                    const float dy = __fsub_rn((float)(y0 + origin_y + (rank >> 1) * 4 + g) + 0.5f, m.y);
                    const uint32_t ub = ubuf(s) + g * 8 * 128 + (((k >> 2) ^ (g << 1)) << 4) + (k & 3) * 4;
                    float m0 = 0.0f, mx = 0.0f, mxx = 0.0f;
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        float u;
                        asm volatile("ld.shared.f32 %0, [%1];" : "=f"(u) : "r"(ub + i * 128));
                        const float dx = __fsub_rn(bx + (float)i, m.x);
                        const float ux = u * dx;
                        m0 += u;
                        mx += ux;
                        mxx = fmaf(ux, dx, mxx);
                    }
                    float my = m0 * dy, mxy = mx * dy, myy = my * dy;
#pragma unroll
                    for (int o = 8; o < 32; o <<= 1) {
                        m0 += __shfl_xor_sync(FULL_MASK, m0, o);
                        mx += __shfl_xor_sync(FULL_MASK, mx, o);
                        my += __shfl_xor_sync(FULL_MASK, my, o);
                        mxx += __shfl_xor_sync(FULL_MASK, mxx, o);
                        mxy += __shfl_xor_sync(FULL_MASK, mxy, o);
                        myy += __shfl_xor_sync(FULL_MASK, myy, o);
                    }
                    float cr = 0.0f, cg = 0.0f, cb = 0.0f;
                    if (RGB) {
                        // dL/dcolour of the entry: sum over the row of w dL/dpixel, w read back from this
                        // block's quadrant of W before the dF transpose reuses the buffer.
                        const int p0 = rank * QPIX + g * 8;
                        const uint32_t wb = fw(s) + w_offset(p0, k);
#pragma unroll
                        for (int i = 0; i < 8; i++) {
                            uint16_t h, l;
                            asm volatile("ld.shared.u16 %0, [%1];" : "=h"(h) : "r"(wb + i * 16));
                            asm volatile("ld.shared.u16 %0, [%1];" : "=h"(l) : "r"(wb + W_BYTES + i * 16));
                            const float w = __uint_as_float((uint32_t)h << 16) + __uint_as_float((uint32_t)l << 16);
                            const float* gp = s_gp[g * 8 + i];
                            cr = fmaf(w, gp[0], cr);
                            cg = fmaf(w, gp[1], cg);
                            cb = fmaf(w, gp[2], cb);
                        }
#pragma unroll
                        for (int o = 8; o < 32; o <<= 1) {
                            cr += __shfl_xor_sync(FULL_MASK, cr, o);
                            cg += __shfl_xor_sync(FULL_MASK, cg, o);
                            cb += __shfl_xor_sync(FULL_MASK, cb, o);
                        }
                    }
                    if (g == 0 && kv) {
                        const int gid = ce.id[k];
                        const float4 q = ce.conic[k];
                        const float o = q.w;
                        const float v[6] = {m0, o * fmaf(q.y, my, q.x * mx), o * fmaf(q.z, my, q.y * mx),
                                            -0.5f * o * mxx, -o * mxy, -0.5f * o * myy};
                        if (v[0] != 0.0f) atomicAdd(grad_opacities + gid, v[0]);
                        if (v[1] != 0.0f) atomicAdd(grad_means2D + 2 * gid, v[1]);
                        if (v[2] != 0.0f) atomicAdd(grad_means2D + 2 * gid + 1, v[2]);
                        if (v[3] != 0.0f) atomicAdd(grad_conics + 3 * gid, v[3]);
                        if (v[4] != 0.0f) atomicAdd(grad_conics + 3 * gid + 1, v[4]);
                        if (v[5] != 0.0f) atomicAdd(grad_conics + 3 * gid + 2, v[5]);
                        if (RGB) {
                            if (cr != 0.0f) atomicAdd(grad_colors + 3 * gid, cr);
                            if (cg != 0.0f) atomicAdd(grad_colors + 3 * gid + 1, cg);
                            if (cb != 0.0f) atomicAdd(grad_colors + 3 * gid + 2, cb);
                        }
                    }
                }
                // This warp is done with the chunk's list entries (the drain warps release them too).
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&s_list_free[e % LIST_SLOTS]);
            }
            if (!fresh) continue;
            if (c >= STAGES && cnt > 0) {
                // Stage s holds chunk c - STAGES's W until its dF MMA has read it; the geometry above
                // read it too, and the group barrier below orders those reads before the stores.
                bool bad = false;
                if (otid == 0) {
                    bad = *(volatile int*)&s_fail ||
                          !tc::mbar_wait_bounded(&s_df_full[s], ((c - STAGES) / STAGES) & 1, WAIT_LIMIT);
                    if (bad) s_fail = 1;
                }
                if (tc::group_sync_count<OPERAND_BAR>(bad) != 0) break;
            }
            if (cnt > 0) {
                // Chunk c's features as bf16 hi + lo (zeros past cnt) into stage s.
                const int k = ow * 8 + (lane >> 2);
                const uint32_t fh = fw(s), fl = fh + K::F_BYTES;
#pragma unroll
                for (int j = 0; j < CK / 16; j++) {
                    const int c4 = j * 4 + (lane & 3);
                    uint32_t h0, l0, h1, l1;
                    split_bf16(fv[j].x, fv[j].y, h0, l0);
                    split_bf16(fv[j].z, fv[j].w, h1, l1);
                    const uint32_t off = (c4 >> 1) * K::F_LBO + k * 16 + (c4 & 1) * 8;
                    st_shared_v2(fh + off, h0, h1);
                    st_shared_v2(fl + off, l0, l1);
                }
            }
            tc::fence_proxy_async();
            tc::fence_before_sync();
            tc::group_sync<OPERAND_BAR>();
            if (otid == 0) tc::mbar_arrive(&s_ready[s]);
            if (cnt == 0) n_real = c;
        }
    } else if (role == Role::Mma) {
        // ------------------------------------------------------------------ MMA warp 13 (one lane)
        // Polls two queues: the dot of the next published chunk, and the dF of the oldest chunk
        // whose four W quadrants have all arrived.
        if (lane == 0) {
            int cd = 0, cf = 0, n_end = -1;
            uint64_t* last_bar = nullptr;
            uint32_t last_par = 0, idle = 0;
            while (n_end < 0 || cf < n_end) {
                if (*(volatile int*)&s_fail) break;
                bool progress = false;
                if (n_end < 0 && tc::mbar_test_wait(&s_ready[cd % STAGES], (cd / STAGES) & 1)) {
                    const int s = cd % STAGES;
                    if (s_list[cd % LIST_SLOTS].count == 0) {
                        n_end = cd;
                    } else {
                        tc::fence_after_sync();
                        const uint32_t fh = fw(s), fl = fh + K::F_BYTES;
#pragma unroll
                        for (int ks = 0; ks < CK / 16; ks++) {
                            const uint32_t ah = tmem + G_TMEM + ks * 8, al = ah + CK / 2;  // A = G from TMEM
                            const uint64_t bh = tc::smem_desc(fh + ks * 2 * K::F_LBO, K::F_LBO, 128);
                            const uint64_t bl = tc::smem_desc(fl + ks * 2 * K::F_LBO, K::F_LBO, 128);
                            const uint32_t d = tmem + s * 32;
                            tc::mma_bf16_ta(d, ah, bh, K::IDESC_DOT, ks > 0 ? 1u : 0u);
                            tc::mma_bf16_ta(d, ah, bl, K::IDESC_DOT, 1u);
                            tc::mma_bf16_ta(d, al, bh, K::IDESC_DOT, 1u);
                        }
                        tc::commit(&s_dot_full[s]);
                        last_bar = &s_dot_full[s];
                        last_par = (cd / STAGES) & 1;
                        cd++;
                    }
                    progress = true;
                }
                // dF of chunk cf overwrites the TMEM columns of chunk cf - STAGES: the drain warps must
                // have read them.
                if (cf < cd &&
                    (cf < STAGES || tc::mbar_test_wait(&s_tmem_free[cf % STAGES], ((cf - STAGES) / STAGES) & 1)) &&
                    tc::mbar_test_wait_cluster(&s_w_full[cf % STAGES], (cf / STAGES) & 1)) {
                    // dF^T of chunk cf = G^T W: A = G^T from TMEM, B = W MN-major (SBO 128 between entry
                    // blocks, LBO 512 between pixel groups).
                    const int s = cf % STAGES;
                    // The peers' quadrants were written by st.async (the generic proxy): order them
                    // before the tensor cores' reads.
                    tc::fence_proxy_async();
                    tc::fence_after_sync();
                    const uint32_t wh = fw(s), wl = wh + W_BYTES;
#pragma unroll
                    for (int ks = 0; ks < PIX / 16; ks++) {
                        const uint32_t ah = tmem + GT_TMEM + ks * 8, al = ah + PIX / 2;
                        const uint64_t bh = tc::smem_desc(wh + ks * 1024, 512, 128);
                        const uint64_t bl = tc::smem_desc(wl + ks * 1024, 512, 128);
                        const uint32_t d = tmem + 128 + s * 32;
                        tc::mma_bf16_ta(d, ah, bh, K::IDESC_DF, ks > 0 ? 1u : 0u);
                        tc::mma_bf16_ta(d, ah, bl, K::IDESC_DF, 1u);
                        tc::mma_bf16_ta(d, al, bh, K::IDESC_DF, 1u);
                    }
                    tc::commit(&s_df_full[s]);
                    last_bar = &s_df_full[s];
                    last_par = (cf / STAGES) & 1;
                    cf++;
                    progress = true;
                }
                if (progress) {
                    idle = 0;
                } else if (++idle > POLL_LIMIT) {
                    s_fail = 1;
                    break;
                }
            }
            if (last_bar != nullptr && !tc::mbar_wait_bounded(last_bar, last_par, WAIT_LIMIT)) s_fail = 1;
        }
    } else if (role == Role::Drain) {
        // ------------------------------------------------------------------ drain warps 14-17
        // Warp q (= warp & 3, its TMEM lane quadrant) has two jobs, polled in turn:
        //  * send: as soon as chunk x's dot is in TMEM, its quadrant q (32 pixels x 32 entries of this
        //    block's channel slice) goes to block q -- into this block's own receive buffer when
        //    q == rank, else by st.async into the peer's.  The owner's buffer of chunk x last held
        //    chunk x - STAGES, which it has walked: the dot of chunk x needed this block's stage,
        //    whose W of chunk x - STAGES came from every block's walk of that chunk.
        //  * drain: chunk e's dF out of TMEM (lane = channel) into dL/dfeatures, one coalesced
        //    128-byte reduction per entry.  The TMEM columns are released as soon as they are read.
        const int q4 = warp & 3;
        const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
        const int cl = q4 * 32 + lane;
        float* const dst = grad_features + c0 + cl;
        // Where this lane's partial goes: owner q4's receive buffer, slice `rank`, pixel `lane`.
        const uint32_t recv_local = recv(0) + rank * RECV_SLICE_BYTES + lane * 128;
        const uint32_t recv_dst = tc::map_shared(recv_local, q4);
        const uint32_t recv_bar = tc::map_shared(tc::smem_addr(&s_recv_full[0]), q4);
        auto poll = [&](uint64_t* bar, uint32_t par) {
            int done = 0;
            if (lane == 0) done = tc::mbar_test_wait(bar, par) ? 1 : 0;
            return __shfl_sync(FULL_MASK, done, 0) != 0;
        };
        int xs = 0, e = 0, n_end = -1;
        uint32_t idle = 0;
        while (n_end < 0 || e < n_end) {
            if (*(volatile int*)&s_fail) break;
            bool progress = false;
            // The list slot of a chunk is released by these warps (and the operand warps) after its
            // drain, so its barrier cannot run a phase ahead of them.
            if (n_end < 0 && poll(&s_list_full[xs % LIST_SLOTS], (xs / LIST_SLOTS) & 1)) {
                if (s_list[xs % LIST_SLOTS].count == 0) {
                    n_end = xs;
                    progress = true;
                } else if (poll(&s_dot_full[xs % STAGES], (xs / STAGES) & 1)) {
                    const int s = xs % STAGES;
                    tc::fence_after_sync();
                    float v[32];
                    tc::tmem_ld32(tmem + lane_base + s * 32, v);
                    tc::fence_before_sync();
                    if (q4 == rank) {
                        const uint32_t d = recv_local + s * K::STAGE_BYTES;
#pragma unroll
                        for (int m8 = 0; m8 < 8; m8++) {
                            const uint32_t seg = (uint32_t)(m8 ^ (lane & 7));
                            st_shared_v4(d + seg * 16, __float_as_uint(v[4 * m8]), __float_as_uint(v[4 * m8 + 1]),
                                         __float_as_uint(v[4 * m8 + 2]), __float_as_uint(v[4 * m8 + 3]));
                        }
                        __syncwarp();
                        if (lane == 0) tc::mbar_arrive_expect_tx(&s_recv_full[s], (CLUSTER - 1) * RECV_SLICE_BYTES);
                    } else {
                        const uint32_t d = recv_dst + s * K::STAGE_BYTES, bar = recv_bar + s * 8;
#pragma unroll
                        for (int m8 = 0; m8 < 8; m8++) {
                            const uint32_t seg = (uint32_t)(m8 ^ (lane & 7));
                            tc::st_async_v4(d + seg * 16, v[4 * m8], v[4 * m8 + 1], v[4 * m8 + 2], v[4 * m8 + 3], bar);
                        }
                    }
                    xs++;
                    progress = true;
                }
            }
            if (e < xs && poll(&s_df_full[e % STAGES], (e / STAGES) & 1)) {
                const int s = e % STAGES;
                const BwdChunk& ce = s_list[e % LIST_SLOTS];
                const int ecnt = ce.count;
                tc::fence_after_sync();
                float v[32];
                tc::tmem_ld32(tmem + lane_base + 128 + s * 32, v);
                tc::fence_before_sync();
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&s_tmem_free[s]);
                if (cl < CK) {
#pragma unroll
                    for (int k = 0; k < KC; k++)
                        if (k < ecnt && v[k] != 0.0f) atomicAdd(dst + (size_t)ce.id[k] * C, v[k]);
                }
                __syncwarp();
                if (lane == 0) tc::mbar_arrive(&s_list_free[e % LIST_SLOTS]);
                e++;
                progress = true;
            }
            if (progress) {
                idle = 0;
            } else if (++idle > POLL_LIMIT) {
                if (lane == 0) s_fail = 1;
                break;
            }
        }
    } else {  // Role::Pixel
        // ------------------------------------------------------------------ pixel warps 0-7
        // Eight threads per pixel of this block's quadrant; thread j takes entries 4j..4j+3.
        const int pq = warp * 4 + (lane >> 3), j = lane & 7;
        const int p = rank * QPIX + pq;
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
        if (RGB) {
            if (inside) {
                gpr = grad_image[3 * pix];
                gpg = grad_image[3 * pix + 1];
                gpb = grad_image[3 * pix + 2];
            }
            bgdot = fmaf(background[2], gpb, fmaf(background[1], gpg, background[0] * gpr));
            if (j == 0) {
                s_gp[pq][0] = gpr;
                s_gp[pq][1] = gpg;
                s_gp[pq][2] = gpb;
            }
        }
        const uint32_t w_off = w_offset(p, 4 * j);
        const uint32_t u_off = pq * 128 + ((j ^ ((pq >> 3) << 1)) << 4);
        const uint32_t r_off = pq * 128 + ((j ^ (pq & 7)) << 4);
        // Every lane polls (each acquires for itself); a timeout on any lane stops the warp.
        auto warp_wait = [&](uint64_t* bar, uint32_t par, bool cluster_scope) {
            bool ok = !*(volatile int*)&s_fail && (cluster_scope ? tc::mbar_wait_cluster_bounded(bar, par, WAIT_LIMIT)
                                                                  : tc::mbar_wait_bounded(bar, par, WAIT_LIMIT));
            ok = __all_sync(FULL_MASK, ok);
            if (!ok && lane == 0) s_fail = 1;
            return ok;
        };

        for (int c = 0;; c++) {
            const int s = c % STAGES;
            const BwdChunk& ch = s_list[c % LIST_SLOTS];
            const uint32_t par = (c / STAGES) & 1;
            // The list slot is released after this warp's walk of the chunk (through the operand warps'
            // geometry), so its barrier cannot run a phase ahead.
            if (!warp_wait(&s_list_full[c % LIST_SLOTS], (c / LIST_SLOTS) & 1, false)) break;
            const int cnt = ch.count;
            if (cnt == 0) break;
            // The four slices' partial dots of the quadrant, sent by the drain warps of the cluster.
            if (!warp_wait(&s_recv_full[s], par, true)) break;

            // Walk: the whole dot of this thread's four entries, summed over the four slices.
            float d[4];
            {
                const uint32_t rb = recv(s) + r_off;
                const float4 t0 = ld_shared_f4(rb), t1 = ld_shared_f4(rb + RECV_SLICE_BYTES);
                const float4 t2 = ld_shared_f4(rb + 2 * RECV_SLICE_BYTES), t3 = ld_shared_f4(rb + 3 * RECV_SLICE_BYTES);
                d[0] = ((t0.x + t1.x) + t2.x) + t3.x;
                d[1] = ((t0.y + t1.y) + t2.y) + t3.y;
                d[2] = ((t0.z + t1.z) + t2.z) + t3.z;
                d[3] = ((t0.w + t1.w) + t2.w) + t3.w;
            }
            const unsigned hits = ch.hits[0];
            float a[4], r[4], g[4], dc[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int k = 4 * j + i;
                const float4 cq = ch.conic[k];
                const float2 m = ch.mean[k];
                const PairAlpha pa = pair_alpha(cx, cy, m.x, m.y, cq.x, cq.y, cq.z, cq.w);
                const float alpha = fminf(MAX_ALPHA, pa.raw);
                const bool ok = ((hits >> k) & 1u) && inside && ch.pos[k] < last && alpha >= MIN_ALPHA;
                a[i] = ok ? alpha : 0.0f;
                r[i] = ok ? __fdividef(1.0f, 1.0f - alpha) : 1.0f;
                // A clamped alpha no longer depends on the gaussian: nothing flows past it.
                g[i] = ok && pa.raw <= MAX_ALPHA ? pa.G : 0.0f;
                dc[i] = 0.0f;
                if (RGB && k < cnt) {  // (slots past cnt may hold stale or never-written entries)
                    const float4 col = ch.col[k];
                    dc[i] = fmaf(col.z, gpb, fmaf(col.y, gpg, col.x * gpr));
                }
            }
            // This segment's map: T_out = P T_in, behind_out = A behind_in + B (the RGB behind: the
            // same A, its own B).
            float P = 1.0f, A = 1.0f, B = 0.0f, Bc = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                P *= r[i];
                B = fmaf(a[i], d[i], (1.0f - a[i]) * B);
                if (RGB) Bc = fmaf(a[i], dc[i], (1.0f - a[i]) * Bc);
                A *= 1.0f - a[i];
            }
            // Inclusive scan over the pixel's eight segments (walk order = lane order), then shift.
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                const float P2 = __shfl_up_sync(FULL_MASK, P, o, 8), A2 = __shfl_up_sync(FULL_MASK, A, o, 8);
                const float B2 = __shfl_up_sync(FULL_MASK, B, o, 8);
                const float Bc2 = RGB ? __shfl_up_sync(FULL_MASK, Bc, o, 8) : 0.0f;
                if (j >= o) {
                    B = fmaf(A, B2, B);
                    if (RGB) Bc = fmaf(A, Bc2, Bc);
                    P = P2 * P;
                    A = A2 * A;
                }
            }
            float Pe = __shfl_up_sync(FULL_MASK, P, 1, 8), Ae = __shfl_up_sync(FULL_MASK, A, 1, 8);
            float Be = __shfl_up_sync(FULL_MASK, B, 1, 8);
            float Bce = RGB ? __shfl_up_sync(FULL_MASK, Bc, 1, 8) : 0.0f;
            if (j == 0) {
                Pe = 1.0f;
                Ae = 1.0f;
                Be = 0.0f;
                Bce = 0.0f;
            }
            float Tk = T * Pe, bh = fmaf(Ae, behind, Be), bhc = fmaf(Ae, behind_rgb, Bce);
            float w[4], u[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                Tk *= r[i];
                float dl = Tk * (d[i] - bh);
                if (RGB) {
                    // The background is seen through T_final, which this entry's alpha scales.
                    dl += Tk * (dc[i] - bhc) - fT * r[i] * bgdot;
                    bhc = fmaf(a[i], dc[i], (1.0f - a[i]) * bhc);
                }
                w[i] = Tk * a[i];
                u[i] = dl * g[i];
                bh = fmaf(a[i], d[i], (1.0f - a[i]) * bh);
            }
            // The pixel's state after the chunk: the last segment's.
            T = __shfl_sync(FULL_MASK, Tk, 7, 8);
            behind = __shfl_sync(FULL_MASK, bh, 7, 8);
            if (RGB) behind_rgb = __shfl_sync(FULL_MASK, bhc, 7, 8);

            // W (bf16 hi + lo) into all four blocks' stage buffers; u for this block's operand warps.
            uint32_t h0, l0, h1, l1;
            split_bf16(w[0], w[1], h0, l0);
            split_bf16(w[2], w[3], h1, l1);
            const uint32_t wl = fw(s) + w_off;
            st_shared_v2(wl, h0, h1);
            st_shared_v2(wl + W_BYTES, l0, l1);
#pragma unroll
            for (int t = 1; t < CLUSTER; t++) {
                const uint32_t peer = (uint32_t)((rank + t) % CLUSTER);
                const uint32_t wr = tc::map_shared(wl, peer);
                const uint32_t bar = tc::map_shared(tc::smem_addr(&s_w_full[s]), peer);
                tc::st_async_v2(wr, h0, h1, bar);
                tc::st_async_v2(wr + W_BYTES, l0, l1, bar);
            }
            st_shared_v4(ubuf(s) + u_off, __float_as_uint(u[0]), __float_as_uint(u[1]), __float_as_uint(u[2]),
                         __float_as_uint(u[3]));
            tc::fence_proxy_async();  // this block's own quadrant of W is read by its tensor cores
            __syncwarp();
            if (lane == 0) {
                if (warp == 0)
                    tc::mbar_arrive_expect_tx(&s_w_full[s], (CLUSTER - 1) * 2 * W_QUAD_BYTES);
                else
                    tc::mbar_arrive(&s_w_full[s]);
                tc::mbar_arrive(&s_walk_done[s]);
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::cluster_sync();  // no block leaves while a peer may still write to its shared memory
    if (s_fail) {
        // After a timeout, stores a peer issued before giving up may still be in flight to this block.
        for (int i = 0; i < 64; i++) __nanosleep(1000);
    }
    if (warp == 0) tc::tmem_dealloc(tmem, TMEM_COLS);
    if (tid == 0 && s_fail) atomicExch(&g_backward_status, HDS_ERR_DEVICE);
}

// lists: half-tile lists to cut first and read (nullptr: the list warps cut them).
template <int CK>
int launch_backward_cluster(int D, int width, int height, int origin_y, const int32_t* tile_ranges, const int32_t* values,
                            const float* means2D, const float* conic4, const float* color_opacity,
                            const float* features, const float* final_T, const int32_t* n_contrib,
                            const float* grad_output, float* grad_features, float* grad_means2D, float* grad_conics,
                            float* grad_opacities, const float* grad_image, const float* background,
                            float* grad_colors, cudaStream_t stream, int helper_every = 0,
                            const HalfTileLists* lists = nullptr) {
    using K = Cfg<CK>;
    const bool rgb = grad_image != nullptr, packed = lists != nullptr;
    auto kernel = rgb ? (packed ? feature_backward_cluster_kernel<CK, true, true> : feature_backward_cluster_kernel<CK, true, false>)
                      : (packed ? feature_backward_cluster_kernel<CK, false, true> : feature_backward_cluster_kernel<CK, false, false>);
    HDS_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, K::SMEM));
    const int tx = tiles_for(width), ty = tiles_for(height);
    const int halves = 2 * tx * ty;
    const int clusters = halves - (helper_every > 1 ? halves / helper_every : 0);
    HalfTileLists l{};
    if (packed) {
        l = *lists;
        int* status = nullptr;
        HDS_CHECK_CUDA(cudaGetSymbolAddress(reinterpret_cast<void**>(&status), g_backward_status));
        cut_half_tile_lists_kernel<<<halves, CUT_THREADS, 0, stream>>>(
            width, height, tx, origin_y, reinterpret_cast<const int2*>(tile_ranges), values,
            reinterpret_cast<const float2*>(means2D), reinterpret_cast<const float4*>(conic4),
            reinterpret_cast<const float4*>(color_opacity), n_contrib, l, status);
        HDS_CHECK_LAUNCH("cut_half_tile_lists_kernel");
    }
    kernel<<<clusters * CLUSTER, THREADS, K::SMEM, stream>>>(
        D, width, height, tx, origin_y, helper_every, reinterpret_cast<const int2*>(tile_ranges), values,
        reinterpret_cast<const float2*>(means2D), reinterpret_cast<const float4*>(conic4),
        reinterpret_cast<const float4*>(color_opacity), features, final_T, n_contrib, grad_output, grad_means2D,
        grad_conics, grad_features, grad_opacities, grad_image, background, grad_colors, l);
    HDS_CHECK_LAUNCH("feature_backward_cluster_kernel");
    return HDS_OK;
}

}  // namespace clus
}  // namespace
}  // namespace hds
