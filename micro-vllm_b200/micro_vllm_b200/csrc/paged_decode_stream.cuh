// Paged GQA decode as one page stream per warp over a queue of work items.
//
// The split grid (paged_decode_mma_kernel) gives every CTA one (split, KV
// head, sequence) and leaves dispatch to the hardware. A per-CTA timeline of
// the Qwen2.5-7B-geometry step on B200 (batch 64, 1k-4k tokens) showed it
// streaming ~7.6 TB/s while every SM holds three CTAs, then losing a fifth of
// the launch to its tail: the SMs that drew short CTAs idle, and an SM left
// with one CTA has only that CTA's eight pages in flight.
//
// Here one CTA per SM runs kStreamWarps independent warps. A work item is a
// run of at most pages_per_split (C) pages of one (sequence, KV head)
// segment: item k of a segment covers pages [k*C, min((k+1)*C, pages)) --
// the split grid's decomposition with equal splits, so results land in the
// same partial layout and the same merge pass combines them. Items are
// numbered in this order:
//   1. every full item (C pages), sequence by sequence, KV head, split;
//   2. each segment's ragged last item, in sequence order;
//   3. one item per KV head of each sequence the decode does not attend
//      (empty: zeros; length out of range: NaN).
// Warps take items in that order from a global counter, so the last items
// taken are the shorter ragged ones. Every CTA derives the numbering from the
// lengths alone (prefix sums), so an index names one item grid-wide. An item
// is a fixed run of pages walked in a fixed order by one warp
// and written to a fixed partial slot, so the result does not depend on
// which warp takes which item: repeated calls are bit-identical.
//
// A warp's TMA ring (kStages pages) runs on across items: the warp holds its
// next item (page IDs, q fragments, the appended row) in registers before
// its current one ends and refills each freed stage with the next page of
// either item. It claims items two at a time, a pair ahead of use: one
// counter shared by the whole grid serialises its atomics (at ~85 claims per
// microsecond, claims of one item taken one item ahead stalled the warps),
// so claiming pairs halves the rate and doubles the time each claim has to
// return. An SM keeps kStreamWarps x kStages pages in flight until the queue
// runs dry.
//
// Per page the math is the split grid's tensor-core tile (WarpPageAttention);
// the fused append (the new K/V row written into the page that holds position
// len - 1 by the warp that reads it), fused RoPE, corrupted-page and bounded
// wait behaviour are the split grid's too.
#pragma once

#include "paged_decode_mma.cuh"

namespace mv {

#ifndef MV_STREAM_WARPS
#define MV_STREAM_WARPS 12
#endif
constexpr int kStreamWarps = MV_STREAM_WARPS;
constexpr int kStreamMaxBatch = 1024;     // sequences whose lengths the CTA tables hold
constexpr int kStreamMaxItemPages = 64;   // pages per item: two page IDs per lane

// 192 KiB of TMA stages per SM, as much in flight as three split-grid CTAs.
template <int D>
struct StreamShape {
    static constexpr int kTileBytes = PageTile<D>::kBytes;
    static constexpr int kStageBytes = 2 * kTileBytes;
    static constexpr int kStages = 192 * 1024 / kStreamWarps / kStageBytes;
    static constexpr int kWarpBytes = kStages * kStageBytes;
    static constexpr int kRingBytes = kStreamWarps * kWarpBytes;
    // After the rings: lengths [B], full-item prefix [B + 1], ragged-item order [B],
    // unattended sequences [B] (int32 each).
    static constexpr int kTableBytes = (4 * kStreamMaxBatch + 1) * 4;
    static constexpr int kSmemBytes = kRingBytes + kTableBytes + 1024;  // + 1 KiB for alignment
    static_assert(kStages >= 2, "at least two stages per warp");
};

// Claim and completion counters of the item queue, at the end of the
// workspace's zero-initialised counter region. Both return to zero at the end
// of every launch: the last warp to finish claiming resets them.
constexpr int kStreamCounterSlots = 2;

// One work item as a warp holds it (warp-uniform fields; id0/id1 per lane).
struct StreamItem {
    int kind;       // 0 attend, 1 empty sequence (zeros), 2 length out of range (NaN), 3 no item
    int b, h;
    int split;      // item index within the segment = partial slot
    int n;          // pages in this item (0 unless kind 0)
    int pages;      // pages of the whole segment
    int len;        // context length
    long long id0;  // physical page of item page `lane` (lanes < n)
    long long id1;  // physical page of item page `lane + 32`
    bool last;      // holds the segment's last page (where the fused append writes)
    bool resolved;  // the flags below are set (the page IDs have been read)
    bool bad;       // a page ID outside the pool, or no RoPE table row: NaN, no loads
    bool append;    // fused append: last page, its ID in the pool, RoPE has its table row
};

struct StreamTables {
    const int* len;     // per sequence: context length (clamped to int32)
    const int* fprefix; // kv_heads x full items of the sequences before b; [B] = all full items
    const int* ragged;  // sequences with a ragged last item, in sequence order
    const int* unused;  // sequences the decode does not attend
    int n_full, n_ragged_items, total;
};

__device__ __forceinline__ StreamItem stream_item(const DecodeParams& p, const StreamTables& t, int index) {
    StreamItem it;
    it.kind = 3;
    it.b = it.h = it.split = it.n = it.pages = it.len = 0;
    it.id0 = it.id1 = 0;
    it.last = it.bad = it.append = false;
    it.resolved = true;
    if (index >= t.total) return it;
    const int C = p.pages_per_split;
    if (index < t.n_full) {
        // Largest b with fprefix[b] <= index; then fprefix[b + 1] > index, so b has full items.
        int lo = 0, hi = p.batch;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (t.fprefix[mid] <= index) lo = mid;
            else hi = mid;
        }
        it.b = lo;
        it.len = t.len[lo];
        it.pages = (it.len + kPageTokens - 1) / kPageTokens;
        const int full = it.pages / C;
        const int r = index - t.fprefix[lo];
        it.h = r / full;
        it.split = r - it.h * full;
        it.n = C;
        it.kind = 0;
    } else if (index < t.n_full + t.n_ragged_items) {
        const int j = index - t.n_full;
        it.b = t.ragged[j / p.kv_heads];
        it.h = j % p.kv_heads;
        it.len = t.len[it.b];
        it.pages = (it.len + kPageTokens - 1) / kPageTokens;
        it.split = it.pages / C;
        it.n = it.pages - it.split * C;
        it.kind = 0;
    } else {
        const int j = index - t.n_full - t.n_ragged_items;
        it.b = t.unused[j / p.kv_heads];
        it.h = j % p.kv_heads;
        it.len = t.len[it.b];
        it.kind = it.len == 0 ? 1 : 2;
    }
    if (it.kind == 0) {
        it.last = static_cast<int64_t>(it.split) * C + it.n == it.pages;
        it.resolved = false;
    }
    return it;
}

// Issue the loads of an item's page IDs (lane i: pages i and i + 32). Nothing
// reads them here, so the warp does not wait for them: stream_item_resolve
// does, just before the item's first page is issued.
__device__ __forceinline__ void stream_item_fetch(const DecodeParams& p, StreamItem& it, int lane) {
    if (it.kind != 0) return;
    const int64_t row = static_cast<int64_t>(it.b) * p.table_stride + static_cast<int64_t>(it.split) * p.pages_per_split;
    if (lane < it.n) it.id0 = load_index(p.block_table, p.table_i64, row + lane);
    if (lane + 32 < it.n) it.id1 = load_index(p.block_table, p.table_i64, row + lane + 32);
}

// The item's corrupted/RoPE flags and whether it carries the fused append
// (every lane calls; once per item). As in the append kernel, the new row is
// written whenever its own page ID is in the pool (and RoPE has a table row
// for it), whatever the other pages of the item hold.
__device__ __forceinline__ void stream_item_resolve(const DecodeParams& p, StreamItem& it, int lane) {
    if (it.resolved) return;
    bool bad = false;
    if (lane < it.n) bad |= it.id0 < 0 || it.id0 >= p.num_blocks;
    if (lane + 32 < it.n) bad |= it.id1 < 0 || it.id1 >= p.num_blocks;
    const bool any_bad = __any_sync(0xffffffffu, bad);
    if (any_bad && lane == 0) report_bad_page_id();
    const bool rope_missing = p.rope_cos && it.len - 1 >= p.rope_rows;
    it.bad = any_bad || rope_missing;
    const int last = it.n - 1;
    const long long last_id = __shfl_sync(0xffffffffu, last < 32 ? it.id0 : it.id1, last & 31);
    it.append = p.new_key && it.last && !rope_missing && last_id >= 0 && last_id < p.num_blocks;
    it.resolved = true;
}

// The new K/V row chunks of the fused append when `it` holds its segment's
// last page (lanes 0..D/8-1: K, the next D/8: V; RoPE applied to K, which
// waits for the loads -- without RoPE nothing waits here).
template <typename T, int D>
__device__ __forceinline__ void stream_new_rows(const DecodeParams& p, const StreamItem& it, int lane,
                                                uint4 (&rows)[(2 * (D / 8) + 31) / 32]) {
    constexpr int kRowChunks = D / 8;
    if (it.kind != 0 || !it.last || !p.new_key) return;
    if (p.rope_cos && it.len - 1 >= p.rope_rows) return;
#pragma unroll
    for (int j = 0; j < (2 * kRowChunks + 31) / 32; ++j) {
        const int c = lane + 32 * j;
        if (c < 2 * kRowChunks) {
            const int which = c >= kRowChunks;
            const int cc = c - which * kRowChunks;
            const int64_t* st = which ? p.new_value_stride : p.new_key_stride;
            const uint4* row = reinterpret_cast<const uint4*>(
                static_cast<const uint16_t*>(which ? p.new_value : p.new_key) + it.b * st[0] + it.h * st[1]);
            rows[j] = row[cc];
            if (p.rope_cos && !which) {
                const int64_t t = static_cast<int64_t>(it.len - 1) * kRowChunks + cc;
                rows[j] = rope_chunk<T>(rows[j], row[cc ^ (kRowChunks / 2)],
                                        reinterpret_cast<const uint4*>(p.rope_cos)[t],
                                        reinterpret_cast<const uint4*>(p.rope_sin)[t], cc < kRowChunks / 2);
            }
        }
    }
}

// Zeros or NaN for the G rows of (b, h), by one warp.
template <typename T>
__device__ void stream_write_constant(const DecodeParams& p, int b, int h, float value, int lane) {
    T* out = static_cast<T*>(p.out);
    const int total = p.group * p.head_dim;
    for (int idx = lane; idx < total; idx += 32) {
        const int g = idx / p.head_dim;
        const int d = idx - g * p.head_dim;
        out[row_out_offset(p, b) + static_cast<int64_t>(h * p.group + g) * p.out_stride_head + d] = from_float<T>(value);
    }
}

// NaN partials for item `split` of (b, h), by one warp.
__device__ void stream_write_partial_nan(const DecodeParams& p, int b, int h, int split, int lane) {
    const float nan = __int_as_float(0x7fffffff);
    const int total = p.group * p.head_dim;
    for (int idx = lane; idx < total; idx += 32) {
        const int g = idx / p.head_dim;
        const int d = idx - g * p.head_dim;
        const int64_t row = (static_cast<int64_t>(b) * p.q_heads + h * p.group + g) * p.max_splits + split;
        p.part_o[row * p.head_dim + d] = nan;
        if (d == 0) p.part_lse[row] = nan;
    }
}

// The fused append for a sequence the decode does not attend, by one warp:
// the new row of head h goes to position len - 1 where the append kernel
// would write it (position inside the table, page inside the pool).
template <typename T>
__device__ void stream_append_direct(const DecodeParams& p, int b, int h, int64_t len, int lane) {
    const int64_t pos = len - 1;
    if (!p.new_key || pos < 0) return;
    if (p.rope_cos && pos >= p.rope_rows) return;
    const int64_t logical = pos / p.block_size;
    if (logical >= p.blocks_per_seq) return;
    const int64_t id = load_index(p.block_table, p.table_i64, b * p.table_stride + logical);
    if (id < 0 || id >= p.num_blocks) {
        if (lane == 0) report_bad_page_id();
        return;
    }
    const int chunks = p.head_dim / 8;
    const int64_t slot = pos - logical * p.block_size;
    for (int c = lane; c < 2 * chunks; c += 32) {
        const int which = c >= chunks;
        const int cc = c - which * chunks;
        const int64_t* st = which ? p.new_value_stride : p.new_key_stride;
        const uint4* row = reinterpret_cast<const uint4*>(
            static_cast<const uint16_t*>(which ? p.new_value : p.new_key) + b * st[0] + h * st[1]);
        uint4 v = row[cc];
        if (p.rope_cos && !which) {
            const int64_t t = pos * chunks + cc;
            v = rope_chunk<T>(v, row[cc ^ (chunks / 2)], reinterpret_cast<const uint4*>(p.rope_cos)[t],
                              reinterpret_cast<const uint4*>(p.rope_sin)[t], cc < chunks / 2);
        }
        uint4* dst = reinterpret_cast<uint4*>(const_cast<uint16_t*>(
                         static_cast<const uint16_t*>(which ? p.v_cache : p.k_cache)) +
                         ((id * p.kv_heads + h) * p.block_size + slot) * p.head_dim) +
                     cc;
        *dst = v;
    }
}

template <typename T, int D>
__global__ void __launch_bounds__(kStreamWarps * 32, 1)
paged_decode_stream_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap) {
    using Shape = StreamShape<D>;
    using Warp = WarpPageAttention<T, D, 1>;
    constexpr int S = Shape::kStages;
    constexpr int kRowChunks = D / 8;
    constexpr int kNewPerLane = (2 * kRowChunks + 31) / 32;

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[kStreamWarps][S];
    __shared__ int counts[2];  // ragged sequences, unattended sequences
    __shared__ int warp_sums[3][kStreamWarps];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tid = threadIdx.x;
    const int C = p.pages_per_split;
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    int* s_len = reinterpret_cast<int*>(smem + Shape::kRingBytes);
    int* s_fprefix = s_len + kStreamMaxBatch;
    int* s_ragged = s_fprefix + kStreamMaxBatch + 1;
    int* s_unused = s_ragged + kStreamMaxBatch;

    const uint32_t bar0 = smem_addr(&bars[warp][0]);
    if (lane == 0) {
#pragma unroll
        for (int st = 0; st < S; ++st) mbar_init(bar0 + 8 * st, 1);
    }
    fence_mbar_init();
    wait_for_prior_grid();
    __syncthreads();

    // ---- tables: every sequence's length, full items per sequence and the
    // lists of sequences with a ragged last item and of sequences not attended,
    // all by prefix sums in sequence order. Every CTA builds the same tables
    // from the same lengths, so an item index names the same item in every CTA
    // (no shared-memory atomics here: their order differs from CTA to CTA).
    constexpr int kPerThread = (kStreamMaxBatch + kStreamWarps * 32 - 1) / (kStreamWarps * 32);
    int my_full[kPerThread];
    unsigned my_bits = 0;  // bit r: sequence r has a ragged item; bit 8 + r: not attended
    int c_full = 0, c_ragged = 0, c_unused = 0;
#pragma unroll
    for (int r = 0; r < kPerThread; ++r) {
        const int b = tid * kPerThread + r;
        my_full[r] = 0;
        if (b < p.batch) {
            const SeqSplit s = seq_split(p, b);
            // The raw length (an unattended sequence's append position needs it).
            s_len[b] = static_cast<int>(s.len < INT32_MIN ? INT32_MIN : (s.len > INT32_MAX ? INT32_MAX : s.len));
            if (s.state == 0) {
                const int pages = static_cast<int>(s.pages);
                my_full[r] = pages / C;
                if (pages % C) {
                    my_bits |= 1u << r;
                    ++c_ragged;
                }
            } else {
                my_bits |= 1u << (8 + r);
                ++c_unused;
            }
            c_full += my_full[r];
        }
    }
    int in_full = c_full, in_ragged = c_ragged, in_unused = c_unused;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int vf = __shfl_up_sync(0xffffffffu, in_full, off);
        const int vr = __shfl_up_sync(0xffffffffu, in_ragged, off);
        const int vu = __shfl_up_sync(0xffffffffu, in_unused, off);
        if (lane >= off) {
            in_full += vf;
            in_ragged += vr;
            in_unused += vu;
        }
    }
    if (lane == 31) {
        warp_sums[0][warp] = in_full;
        warp_sums[1][warp] = in_ragged;
        warp_sums[2][warp] = in_unused;
    }
    __syncthreads();
    int run_full = in_full - c_full, run_ragged = in_ragged - c_ragged, run_unused = in_unused - c_unused;
    for (int v = 0; v < warp; ++v) {
        run_full += warp_sums[0][v];
        run_ragged += warp_sums[1][v];
        run_unused += warp_sums[2][v];
    }
#pragma unroll
    for (int r = 0; r < kPerThread; ++r) {
        const int b = tid * kPerThread + r;
        if (b < p.batch) {
            s_fprefix[b] = run_full * p.kv_heads;
            run_full += my_full[r];
            if (my_bits & (1u << r)) s_ragged[run_ragged++] = b;
            if (my_bits & (1u << (8 + r))) s_unused[run_unused++] = b;
        }
    }
    if (tid == blockDim.x - 1) {
        s_fprefix[p.batch] = run_full * p.kv_heads;
        counts[0] = run_ragged;
        counts[1] = run_unused;
    }
    __syncthreads();
    allow_next_grid();

    StreamTables tables;
    tables.len = s_len;
    tables.fprefix = s_fprefix;
    tables.ragged = s_ragged;
    tables.unused = s_unused;
    tables.n_full = s_fprefix[p.batch];
    tables.n_ragged_items = counts[0] * p.kv_heads;
    tables.total = tables.n_full + tables.n_ragged_items + counts[1] * p.kv_heads;

    // ---- this warp's stream. Its first two items are fixed; later ones come
    // from the claim counter, one item ahead.
    unsigned* claim_counter = p.counters + (kCounterRegionSlots - kStreamCounterSlots);
    unsigned* done_counter = claim_counter + 1;
    const int total_warps = gridDim.x * kStreamWarps;
    const int gw = blockIdx.x * kStreamWarps + warp;
    uint8_t* wsm = smem + warp * Shape::kWarpBytes;
    const uint32_t wsm_addr = smem_addr(wsm);

    StreamItem cur = stream_item(p, tables, gw);
    StreamItem nxt = stream_item(p, tables, gw + total_warps);
    stream_item_fetch(p, cur, lane);
    stream_item_fetch(p, nxt, lane);
    // Items from 2 x total_warps on are claimed in pairs: claim (lane 0) is the
    // first index of the pair the last atomic took (not yet used); second is
    // the unused second item of the pair in use, or -1.
    int claim = tables.total;
    int second = -1;
    if (gw + total_warps < tables.total && lane == 0)
        claim = 2 * total_warps + 2 * static_cast<int>(atomicAdd(claim_counter, 1u));

    Warp w;
    uint32_t cur_q[Warp::KS][1][2];
    uint32_t nxt_q[Warp::KS][1][2];
    uint4 cur_rows[kNewPerLane];
    uint4 nxt_rows[kNewPerLane];
    if (cur.kind == 0) Warp::load_q_frags(p, cur.b, cur.h, lane, cur_q);
    stream_new_rows<T, D>(p, cur, lane, cur_rows);
    if (nxt.kind == 0) Warp::load_q_frags(p, nxt.b, nxt.h, lane, nxt_q);
    stream_new_rows<T, D>(p, nxt, lane, nxt_rows);
    stream_item_resolve(p, cur, lane);

    // Ring positions count this warp's pages across items: position x sits in
    // stage x % S with phase (x / S) & 1. cur's pages start at cur_base.
    uint32_t cur_base = 0;
    uint32_t issued = 0;
    auto issue_next = [&]() {
        // Every lane calls (warp-uniform); lane 0 issues the page at position `issued`.
        const uint32_t x = issued;
        const bool in_cur = x < cur_base + static_cast<uint32_t>(cur.n);
        if (!in_cur) stream_item_resolve(p, nxt, lane);  // the next item's IDs are needed now
        const StreamItem& it = in_cur ? cur : nxt;
        const int j = static_cast<int>(x - cur_base - (in_cur ? 0u : static_cast<uint32_t>(cur.n)));
        const long long id = __shfl_sync(0xffffffffu, j < 32 ? it.id0 : it.id1, j & 31);
        if (lane == 0) {
            const int st = static_cast<int>(x % S);
            const uint32_t bar = bar0 + 8 * st;
            if (!it.bad) {
                const uint32_t dst = wsm_addr + st * Shape::kStageBytes;
                mbar_arrive_expect_tx(bar, Shape::kStageBytes);
                tma_load_5d(dst, &kmap, 0, 0, 0, it.h, static_cast<int>(id), bar);
                tma_load_5d(dst + Shape::kTileBytes, &vmap, 0, 0, 0, it.h, static_cast<int>(id), bar);
            } else {
                // No load for a corrupted item; complete the phase so the ring stays in step.
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
            }
        }
        issued = x + 1;
    };
    // Top the ring up to S pages ahead of cur_base (after an advance). The
    // stages were last read through the generic proxy (ldmatrix, the append's
    // stores): order those reads before the TMA writes.
    auto fill = [&]() {
        const uint32_t limit = cur_base + static_cast<uint32_t>(cur.n) + static_cast<uint32_t>(nxt.n);
        if (issued < limit && issued < cur_base + S) {
            fence_proxy_async_smem();
            __syncwarp();
        }
        while (issued < limit && issued < cur_base + S) issue_next();
    };
    // Initially the ring is empty: issue up to S pages of cur (then nxt).
    fill();

    bool failed = false;
    uint32_t stuck = 0;  // ring position whose wait gave up
    while (cur.kind != 3) {
        if (cur.kind != 0) {
            stream_write_constant<T>(p, cur.b, cur.h, cur.kind == 1 ? 0.0f : __int_as_float(0x7fffffff), lane);
            stream_append_direct<T>(p, cur.b, cur.h, cur.len, lane);
        } else {
#pragma unroll
            for (int ks = 0; ks < Warp::KS; ++ks) w.qf[ks][0][0] = cur_q[ks][0][0], w.qf[ks][0][1] = cur_q[ks][0][1];
            if (p.rope_cos && !cur.bad) w.rope_q(p, cur.len - 1, lane);
            w.reset();
            const int64_t page0 = static_cast<int64_t>(cur.split) * C;
            for (int j = 0; j < cur.n; ++j) {
                const uint32_t x = cur_base + j;
                const int st = static_cast<int>(x % S);
                const bool ok = mbar_wait_bounded(bar0 + 8 * st, (x / S) & 1);
                if (!__all_sync(0xffffffffu, ok)) {
                    failed = true;
                    stuck = x;
                    break;
                }
                const uint32_t kt = wsm_addr + st * Shape::kStageBytes;
                const uint32_t vt = kt + Shape::kTileBytes;
                const int64_t left = cur.len - (page0 + j) * kPageTokens;
                const int valid = left < kPageTokens ? static_cast<int>(left) : kPageTokens;
                if (cur.append && j == cur.n - 1) {
                        // Fused append: the new row into the staged tile (swizzled slot) and the pool.
                        const long long id = __shfl_sync(0xffffffffu, j < 32 ? cur.id0 : cur.id1, j & 31);
                        const int slot = valid - 1;
                        uint8_t* tiles = wsm + st * Shape::kStageBytes;
#pragma unroll
                        for (int q = 0; q < kNewPerLane; ++q) {
                            const int c = lane + 32 * q;
                            if (c < 2 * kRowChunks) {
                                const int which = c >= kRowChunks;
                                const int cc = c - which * kRowChunks;
                                const int r = (cc >> 3) * 16 + slot;
                                if (!cur.bad)
                                    *reinterpret_cast<uint4*>(tiles + which * Shape::kTileBytes + r * 128 +
                                                              (((cc & 7) ^ (r & 7)) << 4)) = cur_rows[q];
                                uint16_t* pool = const_cast<uint16_t*>(
                                    static_cast<const uint16_t*>(which ? p.v_cache : p.k_cache));
                                reinterpret_cast<uint4*>(pool + ((id * p.kv_heads + cur.h) * kPageTokens + slot) * D)[cc] =
                                    cur_rows[q];
                            }
                        }
                        __syncwarp();
                }
                // K fragments -> scores, then V fragments: the stage is read out
                // with one page-half of fragments live at a time.
                float sc[1][2][4];
                uint32_t vf[Warp::KS][4];
                if (!cur.bad) {
                    uint32_t kf[Warp::KS][4];
                    Warp::load_k(kf, kt, lane);
                    w.scores(kf, sc);
                    Warp::load_v(vf, vt, wsm + st * Shape::kStageBytes + Shape::kTileBytes, valid, lane);
                }
                // The page is in registers: refill its stage before the arithmetic.
                const uint32_t limit = cur_base + static_cast<uint32_t>(cur.n) + static_cast<uint32_t>(nxt.n);
                if (issued < limit) {
                    fence_proxy_async_smem();
                    __syncwarp();
                    issue_next();
                }
                if (!cur.bad) w.update(sc, vf, valid, p.scale_log2, lane);
            }
            if (failed) break;
            w.reduce_l();
            const bool single = cur.split == 0 && cur.n == cur.pages;
            if (cur.bad) {
                if (single) stream_write_constant<T>(p, cur.b, cur.h, __int_as_float(0x7fffffff), lane);
                else stream_write_partial_nan(p, cur.b, cur.h, cur.split, lane);
            } else if (single) {
                w.store_final(p, cur.b, cur.h, lane);
            } else {
                const int64_t row0 = (static_cast<int64_t>(cur.b) * p.q_heads + cur.h * p.group) * p.max_splits + cur.split;
                w.store_partial_strided(p.part_o + row0 * D, p.part_lse + row0, static_cast<int64_t>(p.max_splits) * D,
                                        p.max_splits, p.group, lane);
            }
            cur_base += static_cast<uint32_t>(cur.n);
        }

        // Advance: nxt becomes cur; the claimed index becomes nxt; claim the one
        // after. The new nxt's loads are only issued here.
        cur = nxt;
#pragma unroll
        for (int ks = 0; ks < Warp::KS; ++ks) cur_q[ks][0][0] = nxt_q[ks][0][0], cur_q[ks][0][1] = nxt_q[ks][0][1];
#pragma unroll
        for (int q = 0; q < kNewPerLane; ++q) cur_rows[q] = nxt_rows[q];
        stream_item_resolve(p, cur, lane);
        int index;
        if (second >= 0) {
            index = second;
            second = -1;
        } else {
            index = __shfl_sync(0xffffffffu, claim, 0);
            second = index + 1;
            if (index < tables.total && lane == 0)
                claim = 2 * total_warps + 2 * static_cast<int>(atomicAdd(claim_counter, 1u));
        }
        nxt = stream_item(p, tables, index);
        stream_item_fetch(p, nxt, lane);
        if (nxt.kind == 0) Warp::load_q_frags(p, nxt.b, nxt.h, lane, nxt_q);
        stream_new_rows<T, D>(p, nxt, lane, nxt_rows);
        fill();
    }

    if (failed) {
        // Drain the loads in flight (bounded) before the CTA's shared memory goes
        // away; poison what this warp holds (current, next and claimed items).
        for (uint32_t x = stuck; x < issued; ++x) mbar_wait_bounded(bar0 + 8 * (x % S), (x / S) & 1);
        if (lane == 0) atomicOr(&g_device_status, kStatusWaitTimeout);
        const int index = __shfl_sync(0xffffffffu, claim, 0);
        StreamItem held[5] = {cur, nxt, stream_item(p, tables, second >= 0 ? second : tables.total),
                              stream_item(p, tables, index), stream_item(p, tables, index + 1)};
        for (int k = 0; k < 5; ++k) {
            const StreamItem& it = held[k];
            if (it.kind != 0) continue;
            if (it.split == 0 && it.n == it.pages) stream_write_constant<T>(p, it.b, it.h, __int_as_float(0x7fffffff), lane);
            else stream_write_partial_nan(p, it.b, it.h, it.split, lane);
        }
    }
    // This warp claims nothing more. The last warp to get here resets the
    // counters for the next launch (every claim of this launch has been made).
    if (lane == 0) {
        const unsigned old = atomicAdd(done_counter, 1u);
        if (old == static_cast<unsigned>(total_warps) - 1u) {
            *claim_counter = 0u;
            *done_counter = 0u;
        }
    }
}

}  // namespace mv
