// render_features.cu -- C-channel feature blend on tcgen05 tensor cores (split-bf16 contraction).
//
// Restates features.cu:116-346 of the reference (render_features + its host wrapper): every pixel
// blends its tile's sorted list front to back with the same alpha / transmittance walk as the RGB
// pass, and the feature image is out[p, c] = sum_j w[p, j] f[j, c] with w = alpha * T.
//
// Precision.  The contraction runs on kind::f16 tensor cores with every weight and feature split
// into bf16 halves, x = hi + lo + O(2^-17 x), and each product formed as hi*hi + hi*lo + lo*hi (three
// MMAs into one fp32 TMEM accumulator; the dropped lo*lo term is O(2^-16) of the product).  Against
// the FP32 blend the error is ~1e-5 of sum |w f|, inside the 1e-3 absolute feature bound for
// features of any magnitude (one TF32 rounding of each factor, 2^-11, is not: 1.6e-3 on N(0, 1)
// features).  The bf16 pair occupies the bytes one TF32 operand would, and a kind::f16 MMA of
// K = 16 reads what a kind::tf32 MMA of K = 8 reads, so the three products cost 1.5x the operand
// reads of one TF32 contraction.
//
// Blackwell design.  A block owns half a 16x16 tile: 128 pixels, one per TMEM lane.  It runs two
// warp groups that hand chunks of 32 gaussians to each other through a two-stage ring:
//   * producer warps 4-7: warp 4 fills a stage with the next list entries whose opacity-aware box
//     touches the half tile (keeping each one's list position for the contributor count); all four
//     then gather the entries' feature rows with 16-byte loads, split them and store them as the
//     MN-major B operand (channel blocks of 8 x 32 entries, 16 bytes per entry);
//   * pixel warps 0-3: one thread per pixel walks the stage's entries with the oracle's exact FP32
//     arithmetic (a warp skips entries whose box misses its 8 x 4 pixels) and writes its split
//     weights as the K-major A operand; then thread 0 issues 2 x 3 tcgen05.mma (M = 128, N = C,
//     K = 16) into the TMEM accumulators and commits them to the stage's mbarrier.
// The producers run a stage ahead, so gathering, walking and the tensor cores overlap.  The
// accumulators stay in TMEM until the epilogue (tcgen05.ld).  The same walk writes the RGB image,
// final transmittance and contributor count, bit-identical to the RGB kernel.
//
// Every mbarrier wait is bounded; a group that sees a wait run out stops uniformly (the decision is
// taken at a group barrier), records HDS_ERR_DEVICE in g_status (read by hds_device_status), frees
// the block's TMEM and returns.
#include "hds_common.cuh"
#include "tcgen05.cuh"

namespace hds {

__device__ int g_status = 0;

namespace {

constexpr uint32_t WAIT_LIMIT = 1u << 22;
constexpr int STAGES = 2;
constexpr int PIXEL_BAR = 1, PRODUCER_BAR = 2;  // named barriers of the two warp groups

// Operand layouts shared by both forward kernels (bf16, no swizzle; KC = 32 entries per chunk):
//   A (weights, M = 128 pixels x K = 32 entries), K-major: element (p, k) at
//     (k / 8) * A_LBO + (p / 8) * 128 + (p % 8) * 16 + (k % 8) * 2, A_LBO = 2048;
//   B (features, K = 32 entries x N = C channels), MN-major: element (k, n) at
//     (n / 8) * B_SBO + (k / 8) * 128 + (k % 8) * 16 + (n % 8) * 2, B_SBO = 512,
// one copy each for the hi and the lo halves.  A K = 16 step starts 2 * A_LBO into A and 256 bytes
// into B.
constexpr int KC_ENTRIES = 32;
constexpr int A_LBO_BF16 = 2048;
constexpr int A_COPY_BYTES = 128 * KC_ENTRIES * 2;  // one bf16 copy of A: 8 KB
constexpr int B_SBO_BF16 = KC_ENTRIES * 16;          // 512: between 8-channel blocks of B

// A gather item (k, cb) = channels 8 cb .. 8 cb + 7 of entry k, for item index i of 32 * C / 8:
// within a warp, lanes take 8 entries x 4 channel blocks, so that the 32 16-byte stores of a warp hit
// every bank once per wavefront and each entry's 4 lanes read 128 contiguous bytes of its row.
__device__ __forceinline__ int gather_entry(int i) { return (i & 7) | (((i >> 5) & 3) << 3); }
__device__ __forceinline__ int gather_block(int i) { return ((i >> 3) & 3) | ((i >> 7) << 2); }

// Splits eight channels and stores them as one 16-byte row of B's hi and lo copies.
__device__ __forceinline__ void store_split8(uint32_t hi_addr, uint32_t lo_addr, float4 a, float4 b) {
    uint32_t h0, h1, h2, h3, l0, l1, l2, l3;
    tc::split_bf16(a.x, a.y, h0, l0);
    tc::split_bf16(a.z, a.w, h1, l1);
    tc::split_bf16(b.x, b.y, h2, l2);
    tc::split_bf16(b.z, b.w, h3, l3);
    tc::st_shared_v4(hi_addr, h0, h1, h2, h3);
    tc::st_shared_v4(lo_addr, l0, l1, l2, l3);
}

// The three MMAs of one K = 16 step of the split-bf16 product: hi*hi + hi*lo + lo*hi.
__device__ __forceinline__ void mma_split3(uint32_t d, uint64_t a_hi, uint64_t a_lo, uint64_t b_hi, uint64_t b_lo,
                                          uint32_t idesc, uint32_t accumulate) {
    tc::mma_bf16(d, a_hi, b_hi, idesc, accumulate);
    tc::mma_bf16(d, a_hi, b_lo, idesc, 1u);
    tc::mma_bf16(d, a_lo, b_hi, idesc, 1u);
}

template <int C>
struct FwdCfg {
    static constexpr int PIX = 128;
    static constexpr int THREADS = 256;
    static constexpr int KC = KC_ENTRIES;
    static constexpr int N_MMA = C < 256 ? C : 256;
    static constexpr int N_BLOCKS = C / N_MMA;
    static_assert(N_BLOCKS >= 1 && N_BLOCKS * N_MMA == C, "the MMAs must cover every channel");
    static constexpr int TMEM_COLS = C;
    static constexpr int A_BYTES = 2 * A_COPY_BYTES;      // hi + lo
    static constexpr int B_COPY = (C / 8) * B_SBO_BF16;   // one bf16 copy of B
    static constexpr int B_BYTES = 2 * B_COPY;            // hi + lo
    static constexpr int SMEM = STAGES * (A_BYTES + B_BYTES) + 1024;
    static constexpr uint32_t IDESC = tc::idesc_bf16(128, N_MMA, false, true);
    static constexpr int GATHER_ITEMS = KC * (C / 8);     // (entry, 8-channel block) pairs of a chunk
    static_assert(GATHER_ITEMS % 128 == 0, "the producer sweeps must tile the chunk");
    static_assert(C == 32 || C == 64 || C == 128 || C == 256 || C == 512, "unsupported channel count");
};


// One stage's list entries (written by producer warp 4, read by everyone).
struct Chunk {
    int id[32];
    int pos[32];  // position in the tile's list, for the contributor count
    float2 mean[32];
    float2 ext[32];
    float4 conic[32];  // a, b, c, 0
    float4 col[32];    // r, g, b, opacity
    unsigned hits[4];  // bit k: entry k's box touches the 8 x 4 pixel block of pixel warp w
    int count;
};

__device__ __forceinline__ void st_shared_v4f(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

template <int C>
__global__ void __launch_bounds__(256, 1) feature_forward_kernel(
    int width, int height, int tiles_x, int origin_y, const int2* __restrict__ ranges,
    const int32_t* __restrict__ values,
    const float2* __restrict__ means2D, const float4* __restrict__ conic4, const float4* __restrict__ color_opacity,
    const float* __restrict__ features, const float* __restrict__ background, float* __restrict__ feature_image,
    float* __restrict__ final_T, int32_t* __restrict__ n_contrib, float4* __restrict__ image4) {
    using Cfg = FwdCfg<C>;
    extern __shared__ uint8_t smem_raw[];
    __shared__ Chunk s_chunk[STAGES];
    __shared__ uint64_t s_geo_full[STAGES], s_b_full[STAGES], s_mma_done[STAGES];
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail, s_stop;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x >> 1;
    const int x0 = (tile % tiles_x) * TILE;
    const int y0 = (tile / tiles_x) * TILE + (blockIdx.x & 1) * 8;
    if (y0 >= height) return;  // the lower half of a bottom-row tile can lie wholly outside the image

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t a_base = tc::smem_addr(smem);
    const uint32_t b_base = a_base + STAGES * Cfg::A_BYTES;

    if (warp == 0) tc::tmem_alloc(&s_tmem, Cfg::TMEM_COLS);
    if (tid == 0) {
        for (int s = 0; s < STAGES; s++) {
            tc::mbar_init(&s_geo_full[s], 32);
            tc::mbar_init(&s_b_full[s], 128);
            tc::mbar_init(&s_mma_done[s], 1);
        }
        tc::fence_mbar_init();
        s_fail = 0;
        s_stop = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s_tmem;
    const int2 range = ranges[tile];
    const int count = range.y - range.x;

    if (warp >= 4) {
        // ------------------------------------------------------------------ producer warps 4-7
        const int ptid = tid - 128;
        // Pixel-centre rectangle of the half tile.
        const float hx0 = (float)x0 + 0.5f, hx1 = hx0 + 15.0f, hy0 = (float)(y0 + origin_y) + 0.5f, hy1 = hy0 + 7.0f;
        int cursor = 0;
        for (int c = 0;; c++) {
            const int s = c % STAGES;
            Chunk& ch = s_chunk[s];
            // The stage is free once the MMAs of chunk c - STAGES have read it.  Whether to stop is
            // thread 0's view, broadcast by the barrier, so warp 4's lanes never diverge on it.
            bool halt = false;
            if (ptid == 0) {
                if (c >= STAGES && !tc::mbar_wait_bounded(&s_mma_done[s], ((c - STAGES) / STAGES) & 1, WAIT_LIMIT))
                    s_fail = 1;
                halt = *(volatile int*)&s_stop || *(volatile int*)&s_fail;
            }
            const bool stop = tc::group_sync_count<PRODUCER_BAR>(halt) != 0 || cursor >= count;
            if (warp == 4) {
                int filled = 0, cur = cursor;
                if (!stop) {
                    while (filled < Cfg::KC && cur < count) {
                        // Two batches of 32 candidates per round trip to memory.
                        int g[2];
                        float2 m[2], e[2];
                        float4 q[2], col[2];
                        bool hit[2];
#pragma unroll
                        for (int b = 0; b < 2; b++) {
                            const int pos = cur + 32 * b + lane;
                            hit[b] = false;
                            g[b] = 0;
                            m[b] = e[b] = make_float2(0.0f, 0.0f);
                            q[b] = col[b] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                            if (pos < count) {
                                g[b] = values[range.x + pos];
                                m[b] = means2D[g[b]];
                                q[b] = conic4[g[b]];
                                col[b] = color_opacity[g[b]];
                                e[b] = cull_extent(q[b].x, q[b].y, q[b].z, col[b].w);
                                hit[b] = box_hits(m[b], e[b], hx0, hx1, hy0, hy1);
                            }
                        }
#pragma unroll
                        for (int b = 0; b < 2; b++) {
                            if (filled == Cfg::KC || cur >= count) break;
                            const unsigned mask = __ballot_sync(FULL_MASK, hit[b]);
                            const int hits = __popc(mask);
                            const int take = min(hits, Cfg::KC - filled);
                            const int rank = __popc(mask & ((1u << lane) - 1u));
                            if (hit[b] && rank < take) {
                                const int slot = filled + rank;
                                ch.id[slot] = g[b];
                                ch.pos[slot] = cur + lane;
                                ch.mean[slot] = m[b];
                                ch.ext[slot] = e[b];
                                ch.conic[slot] = q[b];
                                ch.col[slot] = col[b];
                            }
                            // When the chunk fills mid-batch, resume right after the last entry taken.
                            cur = take < hits ? cur + nth_set_bit(mask, take - 1) + 1 : cur + 32;
                            filled += take;
                        }
                    }
                }
                if (lane == 0) ch.count = filled;
                __syncwarp();
                {
                    // Which entries touch each pixel warp's 8 x 4 block: the pixel warps test bits.
                    const bool valid = lane < filled;
                    const float2 mm = valid ? ch.mean[lane] : make_float2(0.0f, 0.0f);
                    const float2 ee = valid ? ch.ext[lane] : make_float2(-1e30f, -1e30f);
#pragma unroll
                    for (int w = 0; w < 4; w++) {
                        const float bx0 = (float)(x0 + (w & 1) * 8) + 0.5f;
                        const float by0 = (float)(y0 + origin_y + (w >> 1) * 4) + 0.5f;
                        const unsigned mask =
                            __ballot_sync(FULL_MASK, valid && box_hits(mm, ee, bx0, bx0 + 7.0f, by0, by0 + 3.0f));
                        if (lane == 0) ch.hits[w] = mask;
                    }
                }
                __syncwarp();
                tc::mbar_arrive(&s_geo_full[s]);  // every lane, after its own writes
                cursor = min(cur, count);
            }
            tc::group_sync<PRODUCER_BAR>();  // the chunk's entries (and count) are visible to warps 5-7
            const int valid = ch.count;
            if (valid == 0) break;

            // B operand: each producer thread loads its items' 8-channel pieces (two 16-byte loads
            // each, all issued before the first store), splits them into bf16 hi + lo and stores one
            // 16-byte row of each copy.  Entries past the chunk's count are zero.
            {
                constexpr int PER = Cfg::GATHER_ITEMS / 128;
                const uint32_t b_hi = b_base + s * Cfg::B_BYTES, b_lo = b_hi + Cfg::B_COPY;
                float4 v[PER][2];
#pragma unroll
                for (int u = 0; u < PER; u++) {
                    const int i = u * 128 + ptid, k = gather_entry(i), cb = gather_block(i);
                    v[u][0] = v[u][1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (k < valid) {
                        const float4* row = reinterpret_cast<const float4*>(features + (size_t)ch.id[k] * C) + 2 * cb;
                        v[u][0] = __ldg(row);
                        v[u][1] = __ldg(row + 1);
                    }
                }
#pragma unroll
                for (int u = 0; u < PER; u++) {
                    const int i = u * 128 + ptid, k = gather_entry(i), cb = gather_block(i);
                    const uint32_t off = cb * B_SBO_BF16 + k * 16;
                    store_split8(b_hi + off, b_lo + off, v[u][0], v[u][1]);
                }
            }
            tc::fence_proxy_async();
            tc::mbar_arrive(&s_b_full[s]);
        }
    } else {
        // ------------------------------------------------------------------ pixel warps 0-3
        // Pixel of this thread (= A row = TMEM lane): warp w covers an 8 x 4 block of the half tile.
        const int px = x0 + (warp & 1) * 8 + (lane & 7);
        const int py = y0 + (warp >> 1) * 4 + (lane >> 3);
        const bool inside = px < width && py < height;
        const float cx = (float)px + 0.5f, cy = (float)(py + origin_y) + 0.5f;
        const bool rgb = image4 != nullptr;

        float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f;
        int last = 0;
        bool done = !inside;
        int committed = 0;  // chunks whose MMAs thread 0 issued and committed
        for (int c = 0;; c++) {
            const int s = c % STAGES;
            const Chunk& ch = s_chunk[s];
            bool bad = false;
            if (tid == 0) {
                bad = *(volatile int*)&s_fail;
                if (!bad && !tc::mbar_wait_bounded(&s_geo_full[s], (c / STAGES) & 1, WAIT_LIMIT)) {
                    s_fail = 1;
                    bad = true;
                }
            }
            if (tc::group_sync_count<PIXEL_BAR>(bad) != 0) break;
            const int valid = ch.count;
            if (valid == 0) break;

            // A operand: row p = tid; group g of 8 entries at g * A_LBO + (p / 8) * 128 + (p % 8) * 16 in
            // each of the hi and lo copies.
            const uint32_t a_row = a_base + s * Cfg::A_BYTES + (tid >> 3) * 128 + (tid & 7) * 16;
            const bool warp_done = __all_sync(FULL_MASK, done);
            const unsigned hits_w = ch.hits[warp];  // entries whose box touches this warp's pixels
#pragma unroll 1
            for (int g8 = 0; g8 < Cfg::KC / 8; g8++) {
                float w8[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
                if (!warp_done) {
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        const int k = g8 * 8 + e;
                        if (((hits_w >> k) & 1u) && !done) {
                            const float2 m = ch.mean[k];
                            const float4 q = ch.conic[k];
                            const float4 col = ch.col[k];
                            PairAlpha pa = pair_alpha(cx, cy, m.x, m.y, q.x, q.y, q.z, col.w);
                            float alpha = fminf(MAX_ALPHA, pa.raw);
                            if (!(alpha < MIN_ALPHA)) {
                                float test = T * (1.0f - alpha);
                                if (test < MIN_T) {
                                    done = true;
                                } else {
                                    const float w = alpha * T;
                                    if (rgb) {
                                        ar = fmaf(w, col.x, ar);
                                        ag = fmaf(w, col.y, ag);
                                        ab = fmaf(w, col.z, ab);
                                    }
                                    T = test;
                                    last = ch.pos[k] + 1;
                                    w8[e] = w;
                                }
                            }
                        }
                    }
                }
                uint32_t h[4], l[4];
#pragma unroll
                for (int j = 0; j < 4; j++) tc::split_bf16(w8[2 * j], w8[2 * j + 1], h[j], l[j]);
                tc::st_shared_v4(a_row + g8 * A_LBO_BF16, h[0], h[1], h[2], h[3]);
                tc::st_shared_v4(a_row + A_COPY_BYTES + g8 * A_LBO_BF16, l[0], l[1], l[2], l[3]);
            }
            tc::fence_proxy_async();
            // Every pixel thread has written its A row; tell the producers when all pixels are done.
            if (tc::group_sync_count<PIXEL_BAR>(done) == 128 && tid == 0) *(volatile int*)&s_stop = 1;
            if (tid == 0) {
                if (!tc::mbar_wait_bounded(&s_b_full[s], (c / STAGES) & 1, WAIT_LIMIT)) {
                    s_fail = 1;
                } else {
                    tc::fence_after_sync();
                    const uint32_t a_hi = a_base + s * Cfg::A_BYTES, a_lo = a_hi + A_COPY_BYTES;
                    const uint32_t b_hi = b_base + s * Cfg::B_BYTES, b_lo = b_hi + Cfg::B_COPY;
#pragma unroll
                    for (int ks = 0; ks < Cfg::KC / 16; ks++) {
#pragma unroll
                        for (int nb = 0; nb < Cfg::N_BLOCKS; nb++) {
                            const uint32_t a_off = ks * 2 * A_LBO_BF16;
                            const uint32_t b_off = ks * 256 + nb * (Cfg::N_MMA / 8) * B_SBO_BF16;
                            mma_split3(tmem + nb * Cfg::N_MMA, tc::smem_desc(a_hi + a_off, A_LBO_BF16, 128),
                                       tc::smem_desc(a_lo + a_off, A_LBO_BF16, 128),
                                       tc::smem_desc(b_hi + b_off, 128, B_SBO_BF16),
                                       tc::smem_desc(b_lo + b_off, 128, B_SBO_BF16), Cfg::IDESC,
                                       (c > 0 || ks > 0) ? 1u : 0u);
                        }
                    }
                    tc::commit(&s_mma_done[s]);
                    committed = c + 1;
                }
            }
        }

        // tcgen05 operations complete in issue order: once the last commit arrives, every MMA has
        // finished.  This wait runs on the failure path too, so TMEM is never freed under an MMA.
        bool ok = false;
        if (tid == 0) {
            ok = committed > 0 && tc::mbar_wait_bounded(&s_mma_done[(committed - 1) % STAGES],
                                                        ((committed - 1) / STAGES) & 1, WAIT_LIMIT);
            if (committed > 0 && !ok) s_fail = 1;
            ok = ok && !*(volatile int*)&s_fail;
        }
        // Uniform across the group: it decides whether the warp-collective tcgen05.ld runs.
        const bool have = tc::group_sync_count<PIXEL_BAR>(ok) != 0;
        tc::fence_after_sync();
        const size_t p = (size_t)py * width + px;
        {
            // Lane = pixel in TMEM, channels innermost in the image: each block of 16 columns goes
            // through this warp's 2 KB of the (now idle) A stages, so that every store instruction
            // writes 8 pixels x 64 contiguous bytes instead of 32 scattered 16-byte pieces.  Scratch
            // row r (64 bytes) holds pixel r's 16 channels, its 16-byte quads permuted by (r / 2) % 4
            // so that both the writes and the reads are conflict-free.
            const uint32_t scratch = a_base + warp * 2048;
            const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
            // Reading: lane -> pixel 8 g + lane / 4 of the warp's 32 (an 8 x 4 block), quad lane % 4.
            const int rq = lane & 3;
            float* rdst[4];
            bool rin[4];
#pragma unroll
            for (int g = 0; g < 4; g++) {
                const int r = 8 * g + (lane >> 2);
                const int ex = x0 + (warp & 1) * 8 + (r & 7), ey = y0 + (warp >> 1) * 4 + (r >> 3);
                rin[g] = ex < width && ey < height;
                rdst[g] = feature_image + ((size_t)(rin[g] ? ey : 0) * width + (rin[g] ? ex : 0)) * C + 4 * rq;
            }
#pragma unroll 1
            for (int col = 0; col < C; col += 16) {
                float v[16];
                if (have) {
                    tc::tmem_ld16(lane_addr + col, v);  // warp-collective: every lane executes it
                } else {
#pragma unroll
                    for (int i = 0; i < 16; i++) v[i] = 0.0f;
                }
#pragma unroll
                for (int qd = 0; qd < 4; qd++)
                    st_shared_v4f(scratch + lane * 64 + ((qd ^ ((lane >> 1) & 3)) << 4),
                                  make_float4(v[4 * qd], v[4 * qd + 1], v[4 * qd + 2], v[4 * qd + 3]));
                __syncwarp();
#pragma unroll
                for (int g = 0; g < 4; g++) {
                    const int r = 8 * g + (lane >> 2);
                    float4 o;
                    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                 : "=f"(o.x), "=f"(o.y), "=f"(o.z), "=f"(o.w)
                                 : "r"(scratch + r * 64 + ((rq ^ ((r >> 1) & 3)) << 4)));
                    if (rin[g]) *reinterpret_cast<float4*>(rdst[g] + col) = o;
                }
                __syncwarp();
            }
        }
        if (inside) {
            final_T[p] = T;
            n_contrib[p] = last;
            if (rgb)
                image4[p] = make_float4(fmaf(T, background[0], ar), fmaf(T, background[1], ag),
                                        fmaf(T, background[2], ab), 0.0f);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, Cfg::TMEM_COLS);
    if (tid == 0 && s_fail) atomicExch(&g_status, HDS_ERR_DEVICE);
}

// ----------------------------------------------------------------------------------------------
// Warp-specialised variant for C >= 256, where the C-column accumulator (TMEM) admits one block per
// SM anyway.  Roles (448 threads):
//   * pixel warps 0-7, two threads per pixel: warp w covers 16 pixels of TMEM lane quadrant w & 3 (an
//     8 x 2 block); thread t < 16 and t + 16 share a pixel and each computes the alphas of half of
//     every group of eight entries, swaps them (shfl.xor 16), and both run the walk over all eight
//     with the oracle's exact FP32 operations in list order -- RGB, final T and the contributor count
//     stay bit-identical -- each writing its four split weights (8 bytes of each of A's hi and lo
//     copies) of the K-major A operand;
//   * list warp 8 cuts the tile's list (front to back) into chunks of 32 entries whose box meets the
//     half tile, software-pipelined over three 32-position batches, into a ring of list slots;
//   * gather warps 9-12 copy each chunk's feature rows with 16-byte loads (16 in flight per thread),
//     split them into bf16 hi + lo and store them as the MN-major B operand -- no transposition;
//   * MMA warp 13 (one lane) issues 2 x 3 x C/256 tcgen05.mma per chunk (M = 128, N = 256, K = 16)
//     into the TMEM accumulators, releases the list slot, and after the last chunk tells the pixel
//     warps.
// ----------------------------------------------------------------------------------------------
namespace ws {

constexpr int KC = 32;
constexpr int LIST_SLOTS = 6;
constexpr int PIXEL_WARPS = 8, LIST_WARP = 8, GATHER_WARP0 = 9, GATHER_WARPS = 4, MMA_WARP = 13;
constexpr int THREADS = (MMA_WARP + 1) * 32, PIXEL_THREADS = PIXEL_WARPS * 32, GATHER_THREADS = GATHER_WARPS * 32;
static_assert(LIST_WARP == PIXEL_WARPS && GATHER_WARP0 == LIST_WARP + 1 && MMA_WARP == GATHER_WARP0 + GATHER_WARPS,
              "warp roles must partition the block");
constexpr int PIX_BAR = 1, GATHER_BAR = 2;

enum class Role { Pixel, List, Gather, Mma };
__device__ __forceinline__ Role role_of(int warp) {
    return warp < PIXEL_WARPS ? Role::Pixel
           : warp == LIST_WARP ? Role::List
           : warp < GATHER_WARP0 + GATHER_WARPS ? Role::Gather
                                                 : Role::Mma;
}

template <int C>
struct Cfg {
    static constexpr int STAGES = C >= 512 ? 2 : 3;
    static constexpr int N_MMA = 256;
    static constexpr int N_BLOCKS = C / N_MMA;
    static_assert(N_BLOCKS >= 1 && N_BLOCKS * N_MMA == C, "the MMAs must cover every channel");
    static_assert(KC == KC_ENTRIES, "the operand layouts assume 32 entries per chunk");
    static constexpr int A_BYTES = 2 * A_COPY_BYTES;      // hi + lo (layout above)
    static constexpr int B_COPY = (C / 8) * B_SBO_BF16;   // one bf16 copy of B (layout above)
    static constexpr int B_BYTES = 2 * B_COPY;
    static constexpr int SMEM = STAGES * (A_BYTES + B_BYTES) + 1024;
    static constexpr uint32_t IDESC = tc::idesc_bf16(128, N_MMA, false, true);
    static_assert(C == 256 || C == 512, "the warp-specialised forward is for 256 or 512 channels");
    // Gather items (entry, 8-channel block): each is two float4 loads; GATHER_UNROLL items per thread
    // per sweep keep 2 x GATHER_UNROLL loads in flight, and the sweeps tile the chunk exactly.
    static constexpr int GATHER_ITEMS = KC * (C / 8);
    static constexpr int GATHER_UNROLL = 8;
    static_assert(GATHER_ITEMS % (GATHER_UNROLL * GATHER_THREADS) == 0, "gather sweep must tile the chunk");
};

// One list slot: chunk entries in list order.
struct List {
    int id[KC];
    int pos[KC];
    float2 mean[KC];
    float2 ext[KC];
    float4 conic[KC];  // a, b, c, opacity
    float4 col[KC];    // r, g, b, opacity
    unsigned hits[8];  // bit k: entry k's box touches the 8 x 2 pixel block of pixel warp w
    int count;
};

__device__ __forceinline__ int2 half_tile_pixel(int p) {
    return make_int2(((p >> 5) & 1) * 8 + (p & 7), (p >> 6) * 4 + ((p & 31) >> 3));
}

template <int C>
__global__ void __launch_bounds__(THREADS, 1) feature_forward_ws_kernel(
    int width, int height, int tiles_x, int origin_y, const int2* __restrict__ ranges,
    const int32_t* __restrict__ values,
    const float2* __restrict__ means2D, const float4* __restrict__ conic4, const float4* __restrict__ color_opacity,
    const float* __restrict__ features, const float* __restrict__ background, float* __restrict__ feature_image,
    float* __restrict__ final_T, int32_t* __restrict__ n_contrib, float4* __restrict__ image4) {
    using K = Cfg<C>;
    constexpr int S = K::STAGES;
    extern __shared__ uint8_t smem_raw[];
    __shared__ List s_list[LIST_SLOTS];
    __shared__ uint64_t s_list_full[LIST_SLOTS], s_list_free[LIST_SLOTS];
    __shared__ uint64_t s_a_full[S], s_b_full[S], s_mma_done[S], s_acc_ready;
    __shared__ uint32_t s_tmem;
    __shared__ int s_fail, s_have;
    __shared__ int s_zero_from;  // first chunk walked after every pixel was done (its weights are all zero)
    __shared__ int s_skip[S];  // the stage's weights are all zero: every pixel was done before its chunk

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x >> 1;
    const int x0 = (tile % tiles_x) * TILE;
    const int y0 = (tile / tiles_x) * TILE + (blockIdx.x & 1) * 8;
    if (y0 >= height) return;  // the lower half of a bottom-row tile can lie wholly outside the image

    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t a_base = tc::smem_addr(smem);
    const uint32_t b_base = a_base + S * K::A_BYTES;

    if (warp == 0) tc::tmem_alloc(&s_tmem, C);
    if (tid == 0) {
        for (int i = 0; i < LIST_SLOTS; i++) {
            tc::mbar_init(&s_list_full[i], 1);
            tc::mbar_init(&s_list_free[i], 1);
        }
        for (int i = 0; i < S; i++) {
            tc::mbar_init(&s_a_full[i], 1);
            tc::mbar_init(&s_b_full[i], 1);
            tc::mbar_init(&s_mma_done[i], 1);
        }
        tc::mbar_init(&s_acc_ready, 1);
        tc::fence_mbar_init();
        s_fail = 0;
        s_zero_from = 0x7fffffff;
        s_have = 0;
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = s_tmem;
    const int2 range = ranges[tile];
    const int count = range.y - range.x;
    const Role role = role_of(warp);

    if (role == Role::List) {
        // ---------------------------------------------------------------- list warp
        const float hx0 = (float)x0 + 0.5f, hx1 = hx0 + 15.0f, hy0 = (float)(y0 + origin_y) + 0.5f, hy1 = hy0 + 7.0f;
        auto fetch_id = [&](int b) { return b + lane < count ? values[range.x + b + lane] : -1; };
        auto gather = [&](int g, float2& m, float4& q, float4& col) {
            if (g >= 0) {
                m = means2D[g];
                col = color_opacity[g];
                const float4 cq = conic4[g];
                q = make_float4(cq.x, cq.y, cq.z, col.w);
            }
        };
        // Batches of 32 positions (lane l: position base + l), front to back: A = ids, B = ids and
        // geometry, C = geometry and the hit mask that chunks are cut from.
        int base = 0;
        int base_b = base, id_b = fetch_id(base);
        base += 32;
        int base_a = base, id_a = fetch_id(base);
        base += 32;
        float2 m_b = make_float2(0.0f, 0.0f);
        float4 q_b = make_float4(0.0f, 0.0f, 0.0f, 0.0f), col_b = q_b;
        gather(id_b, m_b, q_b, col_b);
        int base_c = 0, id_c = -1;
        float2 m_c = make_float2(0.0f, 0.0f), e_c = m_c;
        float4 q_c = make_float4(0.0f, 0.0f, 0.0f, 0.0f), col_c = q_c;
        unsigned mask_c = 0;
        bool more = base_b < count;
        for (int c = 0;; c++) {
            const int slot = c % LIST_SLOTS;
            List& ch = s_list[slot];
            bool ok = true;
            if (lane == 0 && c >= LIST_SLOTS) {
                ok = !*(volatile int*)&s_fail &&
                     tc::mbar_wait_bounded(&s_list_free[slot], ((c - LIST_SLOTS) / LIST_SLOTS) & 1, WAIT_LIMIT);
                if (!ok) s_fail = 1;
            }
            if (!__shfl_sync(FULL_MASK, ok, 0)) break;
            // Once every pixel is done, the empty chunk ends the list.
            const bool stop = __shfl_sync(FULL_MASK, *(volatile int*)&s_zero_from, 0) != 0x7fffffff;
            int filled = 0;
            while (!stop && filled < KC) {
                if (mask_c == 0) {
                    if (!more) break;  // list exhausted
                    base_c = base_b;
                    id_c = id_b;
                    m_c = m_b;
                    q_c = q_b;
                    col_c = col_b;
                    e_c = id_c >= 0 ? cull_extent_fast(q_c.x, q_c.y, q_c.z, q_c.w) : make_float2(-1e30f, -1e30f);
                    mask_c = __ballot_sync(FULL_MASK, id_c >= 0 && box_hits(m_c, e_c, hx0, hx1, hy0, hy1));
                    more = base_a < count;
                    base_b = base_a;
                    id_b = id_a;
                    m_b = make_float2(0.0f, 0.0f);
                    q_b = col_b = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    gather(id_b, m_b, q_b, col_b);
                    base_a = base;
                    id_a = fetch_id(base);
                    base += 32;
                    continue;
                }
                const int hits = __popc(mask_c);
                const int take = min(hits, KC - filled);
                const int rank = __popc(mask_c & ((1u << lane) - 1u));
                if (((mask_c >> lane) & 1u) && rank < take) {
                    const int k = filled + rank;
                    ch.id[k] = id_c;
                    ch.pos[k] = base_c + lane;
                    ch.mean[k] = m_c;
                    ch.ext[k] = e_c;
                    ch.conic[k] = q_c;
                    ch.col[k] = col_c;
                }
                if (take == hits) {
                    mask_c = 0;
                } else {
                    const int last_lane = nth_set_bit(mask_c, take - 1);
                    mask_c &= ~((2u << last_lane) - 1u);
                }
                filled += take;
            }
            if (lane == 0) ch.count = filled;
            __syncwarp();
            {
                // Which entries touch each pixel warp's 8 x 2 block: the pixel warps test bits.
                const bool valid = lane < filled;
                const float2 m = valid ? ch.mean[lane] : make_float2(0.0f, 0.0f);
                const float2 e = valid ? ch.ext[lane] : make_float2(-1e30f, -1e30f);
#pragma unroll
                for (int w = 0; w < PIXEL_WARPS; w++) {
                    const float bx0 = (float)(x0 + ((w & 3) & 1) * 8) + 0.5f;
                    const float by0 = (float)(y0 + origin_y + ((w & 3) >> 1) * 4 + (w >> 2) * 2) + 0.5f;
                    const unsigned mask =
                        __ballot_sync(FULL_MASK, valid && box_hits(m, e, bx0, bx0 + 7.0f, by0, by0 + 1.0f));
                    if (lane == 0) ch.hits[w] = mask;
                }
            }
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&s_list_full[slot]);
            if (filled == 0) break;
        }
    } else if (role == Role::Gather) {
        // ---------------------------------------------------------------- gather warps
        const int gtid = tid - GATHER_WARP0 * 32;
        for (int c = 0;; c++) {
            const int s = c % S, slot = c % LIST_SLOTS;
            const List& ch = s_list[slot];
            bool bad = false;
            if (gtid == 0) {
                bad = *(volatile int*)&s_fail ||
                      !tc::mbar_wait_bounded(&s_list_full[slot], (c / LIST_SLOTS) & 1, WAIT_LIMIT);
                // Stage s is free once chunk c - S's MMAs have read it.
                if (!bad && ch.count > 0 && c >= S)
                    bad = !tc::mbar_wait_bounded(&s_mma_done[s], ((c - S) / S) & 1, WAIT_LIMIT);
                if (bad) s_fail = 1;
            }
            if (tc::group_sync_count<GATHER_BAR>(bad, GATHER_THREADS) != 0) break;
            const int cnt = ch.count;
            if (cnt == 0) break;
            // Chunks walked after every pixel was done carry zero weights and their MMAs are skipped.
            // (Only those: the chunk that finished the last pixel is still blended.)
            const bool stopped = tc::group_sync_count<GATHER_BAR>(gtid == 0 && c >= *(volatile int*)&s_zero_from,
                                                                  GATHER_THREADS) != 0;
            // Item i = (entry k, 8-channel block cb) (gather_entry / gather_block); entries past the
            // chunk's count are stored as zeros.
            const uint32_t b_hi = b_base + s * K::B_BYTES, b_lo = b_hi + K::B_COPY;
#pragma unroll 1
            for (int i0 = 0; i0 < (stopped ? 0 : K::GATHER_ITEMS); i0 += K::GATHER_UNROLL * GATHER_THREADS) {
                float4 v[K::GATHER_UNROLL][2];
#pragma unroll
                for (int u = 0; u < K::GATHER_UNROLL; u++) {
                    const int i = i0 + u * GATHER_THREADS + gtid, k = gather_entry(i), cb = gather_block(i);
                    v[u][0] = v[u][1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (k < cnt) {
                        const float4* row = reinterpret_cast<const float4*>(features + (size_t)ch.id[k] * C) + 2 * cb;
                        v[u][0] = __ldg(row);
                        v[u][1] = __ldg(row + 1);
                    }
                }
#pragma unroll
                for (int u = 0; u < K::GATHER_UNROLL; u++) {
                    const int i = i0 + u * GATHER_THREADS + gtid, k = gather_entry(i), cb = gather_block(i);
                    const uint32_t off = cb * B_SBO_BF16 + k * 16;
                    store_split8(b_hi + off, b_lo + off, v[u][0], v[u][1]);
                }
            }
            tc::fence_proxy_async();
            tc::group_sync<GATHER_BAR>(GATHER_THREADS);
            if (gtid == 0) tc::mbar_arrive(&s_b_full[s]);
        }
    } else if (role == Role::Mma) {
        // ---------------------------------------------------------------- MMA warp (one lane)
        if (lane == 0) {
            int committed = 0;
            bool issued = false;  // has any MMA written the accumulators?
            for (int c = 0;; c++) {
                const int s = c % S, slot = c % LIST_SLOTS;
                bool ok = !*(volatile int*)&s_fail &&
                          tc::mbar_wait_bounded(&s_list_full[slot], (c / LIST_SLOTS) & 1, WAIT_LIMIT);
                if (ok && s_list[slot].count == 0) break;
                ok = ok && tc::mbar_wait_bounded(&s_a_full[s], (c / S) & 1, WAIT_LIMIT) &&
                     tc::mbar_wait_bounded(&s_b_full[s], (c / S) & 1, WAIT_LIMIT);
                if (!ok) {
                    s_fail = 1;
                    break;
                }
                tc::fence_after_sync();
                const uint32_t a_hi = a_base + s * K::A_BYTES, a_lo = a_hi + A_COPY_BYTES;
                const uint32_t b_hi = b_base + s * K::B_BYTES, b_lo = b_hi + K::B_COPY;
                const bool skip = *(volatile int*)&s_skip[s];
#pragma unroll
                for (int ks = 0; ks < (skip ? 0 : KC / 16); ks++) {
#pragma unroll
                    for (int nb = 0; nb < K::N_BLOCKS; nb++) {
                        const uint32_t a_off = ks * 2 * A_LBO_BF16;
                        const uint32_t b_off = ks * 256 + nb * (K::N_MMA / 8) * B_SBO_BF16;
                        mma_split3(tmem + nb * K::N_MMA, tc::smem_desc(a_hi + a_off, A_LBO_BF16, 128),
                                   tc::smem_desc(a_lo + a_off, A_LBO_BF16, 128),
                                   tc::smem_desc(b_hi + b_off, 128, B_SBO_BF16),
                                   tc::smem_desc(b_lo + b_off, 128, B_SBO_BF16), K::IDESC,
                                   (issued || ks > 0) ? 1u : 0u);
                    }
                }
                issued = issued || !skip;
                tc::commit(&s_mma_done[s]);  // also when skipped: the stage's phase must advance
                committed = c + 1;
                // Pixels and gathers are done with the chunk's list slot once its MMAs are issued.
                tc::mbar_arrive(&s_list_free[slot]);
            }
            bool ok = committed == 0 ||
                      tc::mbar_wait_bounded(&s_mma_done[(committed - 1) % S], ((committed - 1) / S) & 1, WAIT_LIMIT);
            if (!ok) s_fail = 1;
            s_have = issued && ok;
            tc::fence_before_sync();
            tc::mbar_arrive(&s_acc_ready);
        }
    } else {  // Role::Pixel
        // ---------------------------------------------------------------- pixel warps
        const int quad = warp & 3, half16 = warp >> 2, part = lane >> 4;
        const int p = quad * 32 + half16 * 16 + (lane & 15);
        const int2 lp = half_tile_pixel(p);
        const int px = x0 + lp.x, py = y0 + lp.y;
        const bool inside = px < width && py < height;
        const float cx = (float)px + 0.5f, cy = (float)(py + origin_y) + 0.5f;
        const bool rgb = image4 != nullptr;
        float T = 1.0f, ar = 0.0f, ag = 0.0f, ab = 0.0f;
        int last = 0;
        bool done = !inside;
        bool all_done = false;  // every pixel finished before the current chunk (uniform)
        for (int c = 0;; c++) {
            const int s = c % S, slot = c % LIST_SLOTS;
            const List& ch = s_list[slot];
            bool bad = false;
            if (tid == 0) {
                bad = *(volatile int*)&s_fail ||
                      !tc::mbar_wait_bounded(&s_list_full[slot], (c / LIST_SLOTS) & 1, WAIT_LIMIT);
                // The A stage is free once chunk c - S's MMAs have read it.
                if (!bad && ch.count > 0 && c >= S)
                    bad = !tc::mbar_wait_bounded(&s_mma_done[s], ((c - S) / S) & 1, WAIT_LIMIT);
                if (bad) s_fail = 1;
            }
            if (tc::group_sync_count<PIX_BAR>(bad, PIXEL_THREADS) != 0) break;
            const int cnt = ch.count;
            if (cnt == 0) break;
            // A row of pixel p: entry group g of 8 at g * A_LBO + (p / 8) * 128 + (p % 8) * 16 in each of the
            // hi and lo copies; this thread owns entries 4 part .. 4 part + 3 of each group (8 bytes).
            const uint32_t a_row = a_base + s * K::A_BYTES + (p >> 3) * 128 + (p & 7) * 16 + part * 8;
            const unsigned hits_w = ch.hits[warp];  // entries whose box touches this warp's pixels
#pragma unroll 1
            for (int k0 = 0; k0 < (all_done ? 0 : KC); k0 += 8) {
                const int kb = k0 + 4 * part;
                float w_own[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                bool hit[4];
#pragma unroll
                for (int i = 0; i < 4; i++) hit[i] = (hits_w >> (kb + i)) & 1u;
                const bool any = ((hits_w >> k0) & 0xFFu) != 0;  // uniform per warp
                if (any && !__all_sync(FULL_MASK, done)) {  // uniform per warp
                    float a_own[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float4 q = ch.conic[kb + i];
                        const float2 m = ch.mean[kb + i];
                        const PairAlpha pa = pair_alpha(cx, cy, m.x, m.y, q.x, q.y, q.z, q.w);
                        const float alpha = fminf(MAX_ALPHA, pa.raw);
                        a_own[i] = hit[i] && alpha >= MIN_ALPHA ? alpha : 0.0f;
                    }
                    float a8[8];
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const float a_p = __shfl_xor_sync(FULL_MASK, a_own[i], 16);
                        a8[i] = part ? a_p : a_own[i];
                        a8[i + 4] = part ? a_own[i] : a_p;
                    }
                    // The walk of the oracle, in list order (both threads of the pixel run it).
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        if (a8[i] > 0.0f && !done) {
                            const float test = T * (1.0f - a8[i]);
                            if (test < MIN_T) {
                                done = true;
                            } else {
                                const float w = a8[i] * T;
                                if (rgb) {
                                    const float4 col = ch.col[k0 + i];
                                    ar = fmaf(w, col.x, ar);
                                    ag = fmaf(w, col.y, ag);
                                    ab = fmaf(w, col.z, ab);
                                }
                                T = test;
                                last = ch.pos[k0 + i] + 1;
                                if ((i >> 2) == part) w_own[i & 3] = w;
                            }
                        }
                    }
                }
                uint32_t h0, h1, l0, l1;
                tc::split_bf16(w_own[0], w_own[1], h0, l0);
                tc::split_bf16(w_own[2], w_own[3], h1, l1);
                tc::st_shared_v2(a_row + (k0 >> 3) * A_LBO_BF16, h0, h1);
                tc::st_shared_v2(a_row + A_COPY_BYTES + (k0 >> 3) * A_LBO_BF16, l0, l1);
            }
            tc::fence_proxy_async();
            // Every pixel thread has written its A quads (none when all were done before the chunk:
            // then its MMAs are skipped); tell the list and gather warps when all pixels are done.
            const bool was_done = all_done;
            all_done = tc::group_sync_count<PIX_BAR>(done, PIXEL_THREADS) == PIXEL_THREADS;
            if (tid == 0) {
                s_skip[s] = was_done;
                if (all_done && !was_done) *(volatile int*)&s_zero_from = c + 1;
                tc::mbar_arrive(&s_a_full[s]);
            }
        }

        // Epilogue: once the last MMA has completed, warp w drains TMEM lanes of quadrant w & 3
        // (lane = pixel), columns [half16 * C/2, (half16 + 1) * C/2).
        bool ok = false;
        if (tid == 0) ok = tc::mbar_wait_bounded(&s_acc_ready, 0, WAIT_LIMIT) && *(volatile int*)&s_have;
        const bool have = tc::group_sync_count<PIX_BAR>(ok, PIXEL_THREADS) != 0;
        tc::fence_after_sync();
        {
            // Lane = pixel in TMEM, channels innermost in the image: each block of 16 columns goes
            // through this warp's 2 KB of the (now idle) stage buffers, so that every store
            // instruction writes 8 pixels x 64 contiguous bytes instead of 32 scattered 16-byte pieces.
            // Scratch row r (64 bytes) holds pixel r's 16 channels, its 16-byte quads permuted by
            // (r / 2) % 4 so that both the writes and the reads are conflict-free.
            const uint32_t scratch = a_base + warp * 2048;
            const uint32_t lane_addr = tmem + ((uint32_t)(quad * 32) << 16);
            // Reading: lane -> pixel 8 g + lane / 4 of the warp's 32, quad lane % 4.
            const int rq = lane & 3;
            float* rdst[4];
            bool rin[4];
#pragma unroll
            for (int g = 0; g < 4; g++) {
                const int r = 8 * g + (lane >> 2);
                const int2 le = half_tile_pixel(quad * 32 + r);
                const int ex = x0 + le.x, ey = y0 + le.y;
                rin[g] = ex < width && ey < height;
                rdst[g] = feature_image + ((size_t)(rin[g] ? ey : 0) * width + (rin[g] ? ex : 0)) * C + 4 * rq;
            }
#pragma unroll 1
            for (int col = half16 * (C / 2); col < (half16 + 1) * (C / 2); col += 16) {
                float v[16];
                if (have) {
                    tc::tmem_ld16(lane_addr + col, v);
                } else {
#pragma unroll
                    for (int i = 0; i < 16; i++) v[i] = 0.0f;
                }
#pragma unroll
                for (int qd = 0; qd < 4; qd++)
                    st_shared_v4f(scratch + lane * 64 + ((qd ^ ((lane >> 1) & 3)) << 4),
                                  make_float4(v[4 * qd], v[4 * qd + 1], v[4 * qd + 2], v[4 * qd + 3]));
                __syncwarp();
#pragma unroll
                for (int g = 0; g < 4; g++) {
                    const int r = 8 * g + (lane >> 2);
                    float4 o;
                    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                                 : "=f"(o.x), "=f"(o.y), "=f"(o.z), "=f"(o.w)
                                 : "r"(scratch + r * 64 + ((rq ^ ((r >> 1) & 3)) << 4)));
                    if (rin[g]) *reinterpret_cast<float4*>(rdst[g] + col) = o;
                }
                __syncwarp();
            }
        }
        if (inside && part == 0) {
            const size_t pix = (size_t)py * width + px;
            final_T[pix] = T;
            n_contrib[pix] = last;
            if (rgb)
                image4[pix] = make_float4(fmaf(T, background[0], ar), fmaf(T, background[1], ag),
                                          fmaf(T, background[2], ab), 0.0f);
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, C);
    if (tid == 0 && s_fail) atomicExch(&g_status, HDS_ERR_DEVICE);
}

template <int C>
int launch_forward_ws(int width, int height, int origin_y, const int32_t* tile_ranges, const int32_t* values, const float* means2D,
                      const float* conic4, const float* color_opacity, const float* features,
                      const float* background, float* feature_image, float* final_T, int32_t* n_contrib,
                      float* image4, cudaStream_t stream) {
    auto kernel = feature_forward_ws_kernel<C>;
    HDS_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<C>::SMEM));
    int tx = tiles_for(width), ty = tiles_for(height);
    kernel<<<2 * tx * ty, THREADS, Cfg<C>::SMEM, stream>>>(
        width, height, tx, origin_y, reinterpret_cast<const int2*>(tile_ranges), values,
        reinterpret_cast<const float2*>(means2D),
        reinterpret_cast<const float4*>(conic4), reinterpret_cast<const float4*>(color_opacity), features, background,
        feature_image, final_T, n_contrib, reinterpret_cast<float4*>(image4));
    HDS_CHECK_LAUNCH("feature_forward_ws_kernel");
    return HDS_OK;
}

}  // namespace ws

template <int C>
int launch_forward(int width, int height, int origin_y, const int32_t* tile_ranges, const int32_t* values, const float* means2D,
                   const float* conic4, const float* color_opacity, const float* features, const float* background,
                   float* feature_image, float* final_T, int32_t* n_contrib, float* image4, cudaStream_t stream) {
    using Cfg = FwdCfg<C>;
    auto kernel = feature_forward_kernel<C>;
    HDS_CHECK_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM));
    int tx = tiles_for(width), ty = tiles_for(height);
    kernel<<<2 * tx * ty, Cfg::THREADS, Cfg::SMEM, stream>>>(
        width, height, tx, origin_y, reinterpret_cast<const int2*>(tile_ranges), values,
        reinterpret_cast<const float2*>(means2D),
        reinterpret_cast<const float4*>(conic4), reinterpret_cast<const float4*>(color_opacity), features, background,
        feature_image, final_T, n_contrib, reinterpret_cast<float4*>(image4));
    HDS_CHECK_LAUNCH("feature_forward_kernel");
    return HDS_OK;
}

}  // namespace
}  // namespace hds

using namespace hds;

extern "C" int hds_render_features_forward(int n, int channels, int width, int height, int origin_y,
                                           const int32_t* tile_ranges,
                                           const int32_t* values_sorted, const float* means2D, const float* conic4,
                                           const float* color_opacity, const float* features, const float* background,
                                           float* feature_image, float* final_T, int32_t* n_contrib, float* image4,
                                           hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(n >= 0 && width > 0 && height > 0, HDS_ERR_INVALID, "rasterize_features: bad sizes");
    HDS_REQUIRE(origin_y >= 0 && origin_y % TILE == 0, HDS_ERR_INVALID,
                "rasterize_features: origin_y %d must be a non-negative multiple of 16", origin_y);
    HDS_REQUIRE((int64_t)channels * width * height <= INT32_MAX, HDS_ERR_TOO_LARGE,
                "a %dx%d image of %d channels overflows the feature kernels' int indices", width, height, channels);
    HDS_REQUIRE(((uintptr_t)features & 15) == 0 && ((uintptr_t)feature_image & 15) == 0, HDS_ERR_INVALID,
                "rasterize_features: features and feature_image must be 16-byte aligned");
    HDS_REQUIRE(image4 == nullptr || (background != nullptr && ((uintptr_t)image4 & 15) == 0), HDS_ERR_INVALID,
                "rasterize_features: the fused RGB output needs a background and 16-byte alignment");
    switch (channels) {
        case 32: return launch_forward<32>(width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, background, feature_image, final_T, n_contrib, image4, stream);
        case 64: return launch_forward<64>(width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, background, feature_image, final_T, n_contrib, image4, stream);
        case 128: return launch_forward<128>(width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, background, feature_image, final_T, n_contrib, image4, stream);
        case 256: return ws::launch_forward_ws<256>(width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, background, feature_image, final_T, n_contrib, image4, stream);
        case 512: return ws::launch_forward_ws<512>(width, height, origin_y, tile_ranges, values_sorted, means2D, conic4, color_opacity, features, background, feature_image, final_T, n_contrib, image4, stream);
        default:
            set_error("features must have 32, 64, 128, 256 or 512 channels, got %d", channels);
            return HDS_ERR_UNSUPPORTED;
    }
}

extern "C" int hds_device_status(int* status, hds_stream_t stream) {
    clear_error();
    HDS_REQUIRE(status != nullptr, HDS_ERR_INVALID, "device_status: null output");
    int zero = 0, forward = 0, backward = 0;
    HDS_CHECK_CUDA(cudaMemcpyFromSymbolAsync(&forward, g_status, sizeof(int), 0, cudaMemcpyDeviceToHost, stream));
    HDS_CHECK_CUDA(cudaMemcpyToSymbolAsync(g_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, stream));
    if (int rc = read_and_clear_backward_status(&backward, stream)) return rc;
    HDS_CHECK_CUDA(cudaStreamSynchronize(stream));
    *status = forward ? forward : backward;
    return HDS_OK;
}
