// feature_bwd_common.cuh -- pieces shared by the two feature-backward kernels (one block per
// half tile and channel slice, and the four-block cluster that walks each half tile once): the
// chunk of list entries a list warp hands to the walk, the bf16 hi + lo split of the tensor-core
// operands, and the list warp itself.
#pragma once

#include <cuda_bf16.h>

#include "hds_common.cuh"
#include "tcgen05.cuh"

namespace hds {
namespace fbwd {

constexpr uint32_t WAIT_LIMIT = 1u << 22;
constexpr int KC = 32;         // list entries per chunk (the N of both MMAs)
constexpr int PIX = 128;       // pixels per half tile (the TMEM lanes of the dot)
constexpr int LIST_SLOTS = 6;  // list ring: the list warp runs up to three chunks past the operand stages

using tc::split_bf16;
using tc::st_shared_v2;
using tc::st_shared_v4;

// Pixel p (p < 128, the TMEM lane order) of the 16 x 8 half tile: quadrant p/32 is an 8 x 4 block.
__device__ __forceinline__ int2 half_tile_pixel(int p) {
    return make_int2(((p >> 5) & 1) * 8 + (p & 7), (p >> 6) * 4 + ((p & 31) >> 3));
}

// One stage's list entries, in walk order (descending list position).
struct BwdChunk {
    int id[KC];
    int pos[KC];
    float2 mean[KC];
    float2 ext[KC];
    float4 conic[KC];  // a, b, c, opacity
    float4 col[KC];    // r, g, b, opacity (filled when the walk carries the RGB terms)
    unsigned hits[8];  // bit k: entry k's box touches pixel group w (the kernel defines the groups)
    int count;
};

// The list warp: fills s_list[c % LIST_SLOTS] with chunk c of the half tile's entries whose
// opacity-aware box touches the half tile, arrives on s_list_full[slot], and ends with an empty
// chunk.  mark_hits(ch, filled) runs on the whole warp once a chunk is filled and records the
// per-group hit masks.  A slot is refilled only after s_list_free[slot] completes.
template <bool RGB, class MarkHits>
__device__ __forceinline__ void list_producer(int lane, int x0, int y0, int origin_y, int width, int height, int2 range,
                                              const int32_t* __restrict__ values,
                                              const float2* __restrict__ means2D,
                                              const float4* __restrict__ conic4,
                                              const float4* __restrict__ color_opacity,
                                              const int32_t* __restrict__ n_contrib, BwdChunk* s_list,
                                              uint64_t* s_list_full, uint64_t* s_list_free, int* s_fail_ptr,
                                              MarkHits&& mark_hits) {
    int& s_fail = *s_fail_ptr;
    // Walks the tile's list back to front in batches of 32 positions (lane l: position
    // top - 1 - l), software-pipelined over three batches: the sorted ids of batch A, the
    // gathered means / conics / opacities of batch B, and the hit mask of batch C that chunks
    // are cut from.  Hits left over when a chunk fills stay in C's mask for the next chunk.
    // Entries past every pixel's last contributor cannot contribute: start there.
    int m = 0;
#pragma unroll
    for (int q = 0; q < 4; q++) {
        const int2 lp = half_tile_pixel(q * 32 + lane);
        const int px = x0 + lp.x, py = y0 + lp.y;
        if (px < width && py < height) m = max(m, n_contrib[(size_t)py * width + px]);
    }
    int top = min(range.y - range.x, __reduce_max_sync(FULL_MASK, m));
    const float hx0 = (float)x0 + 0.5f, hx1 = hx0 + 15.0f, hy0 = (float)(y0 + origin_y) + 0.5f, hy1 = hy0 + 7.0f;
    auto fetch_id = [&](int t) { return t - 1 - lane >= 0 ? values[range.x + t - 1 - lane] : -1; };
    // Batch A: ids only.  Batch B: ids and gathered geometry.  Batch C: geometry and hits.
    int top_a = top, id_a = fetch_id(top);
    top -= 32;
    int top_b = top, id_b = fetch_id(top);
    top -= 32;
    float2 m_b = make_float2(0.0f, 0.0f);
    float4 q_b = make_float4(0.0f, 0.0f, 0.0f, 0.0f), col_b = q_b;
    auto gather = [&](int g, float2& mm, float4& qq, float4& cc) {
        if (g >= 0) {
            mm = means2D[g];
            const float4 cq = conic4[g];
            cc = color_opacity[g];
            qq = make_float4(cq.x, cq.y, cq.z, cc.w);
        }
    };
    // Prime: B <- first batch (gathered), A <- second batch.
    {
        const int t = top_a, i = id_a;
        top_a = top_b;
        id_a = id_b;
        top_b = t;
        id_b = i;
        gather(id_b, m_b, q_b, col_b);
    }
    int top_c = 0, id_c = -1;
    float2 m_c = make_float2(0.0f, 0.0f), e_c = make_float2(0.0f, 0.0f);
    float4 q_c = make_float4(0.0f, 0.0f, 0.0f, 0.0f), col_c = q_c;
    unsigned mask_c = 0;
    bool more = top_b > 0;  // does batch B hold any position?
    for (int c = 0;; c++) {
        const int slot = c % LIST_SLOTS;
        BwdChunk& ch = s_list[slot];
        if (c >= LIST_SLOTS) {  // the slot's previous chunk must be drained
            bool ok = true;
            if (lane == 0) {
                ok = !*(volatile int*)&s_fail &&
                     tc::mbar_wait_bounded(&s_list_free[slot], ((c - LIST_SLOTS) / LIST_SLOTS) & 1, WAIT_LIMIT);
                if (!ok) s_fail = 1;
            }
            if (!__shfl_sync(FULL_MASK, ok, 0)) break;
        }
        int filled = 0;
        while (filled < KC) {
            if (mask_c == 0) {
                if (!more) break;  // list exhausted
                // Promote B to C (its gathers were issued a batch ago), A to B, and fetch a new A.
                top_c = top_b;
                id_c = id_b;
                m_c = m_b;
                q_c = q_b;
                col_c = col_b;
                e_c = id_c >= 0 ? cull_extent_fast(q_c.x, q_c.y, q_c.z, q_c.w) : make_float2(-1e30f, -1e30f);
                mask_c = __ballot_sync(FULL_MASK, id_c >= 0 && box_hits(m_c, e_c, hx0, hx1, hy0, hy1));
                more = top_a > 0;
                top_b = top_a;
                id_b = id_a;
                m_b = make_float2(0.0f, 0.0f);
                q_b = col_b = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                gather(id_b, m_b, q_b, col_b);
                top_a = top;
                id_a = fetch_id(top);
                top -= 32;
                continue;
            }
            const int hits = __popc(mask_c);
            const int take = min(hits, KC - filled);
            const int rank = __popc(mask_c & ((1u << lane) - 1u));
            if (((mask_c >> lane) & 1u) && rank < take) {
                const int k = filled + rank;
                ch.id[k] = id_c;
                ch.pos[k] = top_c - 1 - lane;
                ch.mean[k] = m_c;
                ch.ext[k] = e_c;
                ch.conic[k] = q_c;
                if (RGB) ch.col[k] = col_c;
            }
            // Clear the taken bits (the lowest `take` set bits: descending positions).
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
        mark_hits(ch, filled);
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&s_list_full[slot]);
        if (filled == 0) break;  // the empty chunk ends the list
    }
}

// ---------------------------------------------------------------------------------------------
// Half-tile lists cut ahead of the walk
// ---------------------------------------------------------------------------------------------
// The list warp above cuts a half tile's chunks while the walk waits for them: a chain of dependent
// loads (sorted ids, then the gaussians' geometry) and a box test per tile entry, once per block.
// cut_half_tile_lists_kernel does the same cut for every half tile at once, ahead of the backward:
// half tile h (tile h >> 1, rows 8 (h & 1) ..+8) of a tile whose list is [r0, r1) keeps its entries
// with list position below the half tile's last contributor whose opacity-aware box touches the
// half tile, in ascending position, at slots [2 r0 + (h & 1)(r1 - r0), ...) of three arrays -- head
// (id, position, mean x, mean y as bits), conic (a, b, c, opacity) and the colour_opacity row --
// with count[h] entries.  A frame of P pairs needs 2 P slots.  The list warp then only streams them
// (list_reader); the chunks, and so every sum, are the ones list_producer cuts.
struct HalfTileLists {
    int4* head;
    float4* conic;
    float4* col;
    int* count;
    int64_t capacity;  // slots
};

__host__ __device__ inline size_t half_tile_counts_bytes(int tiles) { return ((size_t)8 * tiles + 255) & ~(size_t)255; }
__host__ __device__ inline size_t half_tile_lists_bytes(int64_t pairs, int tiles) {
    return half_tile_counts_bytes(tiles) + (size_t)48 * 2 * (size_t)pairs;
}
// The lists laid out in a workspace of `bytes` bytes (256-byte aligned); capacity 0 when too small.
inline HalfTileLists half_tile_lists_in(void* ws, size_t bytes, int tiles) {
    HalfTileLists l{};
    const size_t head = half_tile_counts_bytes(tiles);
    if (ws == nullptr || bytes < head) return l;
    const int64_t cap = (int64_t)((bytes - head) / 48);
    uint8_t* base = static_cast<uint8_t*>(ws);
    l.count = reinterpret_cast<int*>(base);
    l.head = reinterpret_cast<int4*>(base + head);
    l.conic = reinterpret_cast<float4*>(base + head + (size_t)16 * cap);
    l.col = reinterpret_cast<float4*>(base + head + (size_t)32 * cap);
    l.capacity = cap;
    return l;
}

constexpr int CUT_THREADS = 128;

// One block per half tile; 128 list positions per round, compacted in position order.  A half tile
// whose slots would pass the capacity records HDS_ERR_TOO_LARGE in *status and keeps no entry.
__global__ void __launch_bounds__(CUT_THREADS) cut_half_tile_lists_kernel(
    int width, int height, int tiles_x, int origin_y, const int2* __restrict__ ranges,
    const int32_t* __restrict__ values, const float2* __restrict__ means2D, const float4* __restrict__ conic4,
    const float4* __restrict__ color_opacity, const int32_t* __restrict__ n_contrib, HalfTileLists lists,
    int* status) {
    __shared__ int s_top, s_warp[CUT_THREADS / 32];
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int tile = h >> 1;
    const int x0 = (tile % tiles_x) * TILE, y0 = (tile / tiles_x) * TILE + (h & 1) * 8;
    if (y0 >= height) {  // the lower half of a bottom-row tile
        if (tid == 0) lists.count[h] = 0;
        return;
    }
    const int2 range = ranges[tile];
    const int len = range.y - range.x;
    const int64_t base = 2 * (int64_t)range.x + (h & 1) * (int64_t)len;
    if (2 * (int64_t)range.y > lists.capacity) {
        if (tid == 0) {
            lists.count[h] = 0;
            atomicExch(status, HDS_ERR_TOO_LARGE);
        }
        return;
    }
    // The half tile's last contributor (its 128 pixels, one per thread).
    if (tid == 0) s_top = 0;
    __syncthreads();
    {
        const int2 lp = half_tile_pixel(tid);
        const int px = x0 + lp.x, py = y0 + lp.y;
        int m = px < width && py < height ? n_contrib[(size_t)py * width + px] : 0;
        m = __reduce_max_sync(FULL_MASK, m);
        if (lane == 0) atomicMax(&s_top, m);
    }
    __syncthreads();
    const int top = min(len, s_top);
    const float hx0 = (float)x0 + 0.5f, hx1 = hx0 + 15.0f, hy0 = (float)(y0 + origin_y) + 0.5f, hy1 = hy0 + 7.0f;
    int written = 0;
    for (int t0 = 0; t0 < top; t0 += CUT_THREADS) {
        const int t = t0 + tid;
        const int id = t < top ? values[range.x + t] : -1;
        float2 m = make_float2(0.0f, 0.0f);
        float4 q = make_float4(0.0f, 0.0f, 0.0f, 0.0f), co = q;
        bool hit = false;
        if (id >= 0) {
            m = means2D[id];
            q = conic4[id];
            co = color_opacity[id];
            hit = box_hits(m, cull_extent_fast(q.x, q.y, q.z, co.w), hx0, hx1, hy0, hy1);
        }
        const unsigned ballot = __ballot_sync(FULL_MASK, hit);
        if (lane == 0) s_warp[warp] = __popc(ballot);
        __syncthreads();
        int before = written, total = written;
#pragma unroll
        for (int w = 0; w < CUT_THREADS / 32; w++) {
            const int c = s_warp[w];
            before += w < warp ? c : 0;
            total += c;
        }
        if (hit) {
            const int64_t slot = base + before + __popc(ballot & ((1u << lane) - 1u));
            lists.head[slot] = make_int4(id, t, __float_as_int(m.x), __float_as_int(m.y));
            lists.conic[slot] = make_float4(q.x, q.y, q.z, co.w);
            lists.col[slot] = co;
        }
        written = total;
        __syncthreads();  // s_warp is rewritten next round
    }
    if (tid == 0) lists.count[h] = written;
}

// The list warp over cut half-tile lists: the same chunks as list_producer (entries in descending
// position, KC per chunk, then an empty chunk), read as coalesced rows with the next chunk's loads
// in flight while the current one is stored.
template <bool RGB, class MarkHits>
__device__ __forceinline__ void list_reader(int lane, int h, int2 range, const HalfTileLists& lists, BwdChunk* s_list,
                                            uint64_t* s_list_full, uint64_t* s_list_free, int* s_fail_ptr,
                                            MarkHits&& mark_hits) {
    int& s_fail = *s_fail_ptr;
    const int n = lists.count[h];
    const int64_t base = 2 * (int64_t)range.x + (h & 1) * (int64_t)(range.y - range.x);
    auto fetch = [&](int c, int4& hd, float4& q, float4& co) {
        const int i = n - 1 - KC * c - lane;  // entry `lane` of chunk c
        if (i >= 0) {
            hd = lists.head[base + i];
            q = lists.conic[base + i];
            if (RGB) co = lists.col[base + i];
        }
    };
    int4 hd = make_int4(-1, 0, 0, 0);
    float4 q = make_float4(0.0f, 0.0f, 0.0f, 0.0f), co = q;
    fetch(0, hd, q, co);
    for (int c = 0;; c++) {
        const int slot = c % LIST_SLOTS;
        BwdChunk& ch = s_list[slot];
        const int filled = max(0, min(KC, n - KC * c));
        int4 hd_next = make_int4(-1, 0, 0, 0);
        float4 q_next = make_float4(0.0f, 0.0f, 0.0f, 0.0f), co_next = q_next;
        if (filled == KC) fetch(c + 1, hd_next, q_next, co_next);
        if (c >= LIST_SLOTS) {  // the slot's previous chunk must be drained
            bool ok = true;
            if (lane == 0) {
                ok = !*(volatile int*)&s_fail &&
                     tc::mbar_wait_bounded(&s_list_free[slot], ((c - LIST_SLOTS) / LIST_SLOTS) & 1, WAIT_LIMIT);
                if (!ok) s_fail = 1;
            }
            if (!__shfl_sync(FULL_MASK, ok, 0)) break;
        }
        if (lane < filled) {
            ch.id[lane] = hd.x;
            ch.pos[lane] = hd.y;
            ch.mean[lane] = make_float2(__int_as_float(hd.z), __int_as_float(hd.w));
            ch.ext[lane] = cull_extent_fast(q.x, q.y, q.z, q.w);
            ch.conic[lane] = q;
            if (RGB) ch.col[lane] = co;
        }
        if (lane == 0) ch.count = filled;
        __syncwarp();
        mark_hits(ch, filled);
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&s_list_full[slot]);
        if (filled == 0) break;  // the empty chunk ends the list
        hd = hd_next;
        q = q_next;
        co = co_next;
    }
}

}  // namespace fbwd
}  // namespace hds
