// Attention of a chunk of T new tokens per sequence over its pages, as query
// tiles on tensor cores (FlashAttention-2 style, mma.sync, TMA page staging).
//
// Query rows of one (sequence b, KV head h): r = t * G + g for chunk token t
// and query head h*G + g; row r attends the first len - (T - 1 - t) tokens
// (its causal prefix). A CTA owns 64 rows (4 warps x 16) and one split of the
// pages, and streams each page once for all its rows through a shared TMA
// ring: thread 0 issues the first kStages pages, then, after each page, refills
// the stage of the page before it once every warp has released that one (so
// it rarely waits), keeping kStages - 1 pages in flight. Per page and warp:
//   S[16 rows, 16 tok] = Q[16, D] . K_page^T      mma m16n8k16, B = K via ldmatrix
//   per-row causal mask, online softmax in the exp2 domain (quad shuffles)
//   O[16 rows, D]     += P[16, 16 tok] . V_page    mma m16n8k16, A = P from S's
//                                                    accumulators, B = V via ldmatrix.trans
// Four warps of at most 168 registers: three CTAs per SM (a fifth, producer
// warp would put three warps on one scheduler and halve that).
// Results use the decode path's row format: a row whose context fits one split
// is written as output, others as normalised partials + log2-sum-exp at part
// row (z * q_heads + hq) * max_splits + split with z = b * T + t, merged by the
// decode path's merge kernel -- the same numbers the row-per-token form gives,
// up to summation order.
#pragma once

#include "mv_device.cuh"

namespace mv {

constexpr int kChunkRows = 64;        // query rows per CTA
constexpr int kChunkWarps = 4;        // 16 rows each
constexpr int kChunkThreads = kChunkWarps * 32;
constexpr int kChunkMaxPages = 128;   // pages of one split (their IDs are staged in shared memory)
constexpr int kChunkMaxStages = 8;

template <int D>
struct ChunkShape {
    static constexpr int kStages = D == 64 ? 8 : 6;
    static constexpr int kTileBytes = 16 * D * 2;  // one K (or V) page of one head
    static constexpr int kStageBytes = 2 * kTileBytes;
    static constexpr int kSmemBytes = kStages * kStageBytes + 1024;
};

// State of one query row of a chunk (seq_split's rules for row z).
struct ChunkRow {
    int64_t len;    // tokens the row attends
    int state;      // 0 attend, 1 empty (zeros), 2 invalid (NaN), 3 no row (padding)
    int splits;
};

__device__ __forceinline__ ChunkRow chunk_row(const DecodeParams& p, int b, int rr, int64_t seq_len) {
    ChunkRow c;
    c.len = 0;
    c.splits = 1;
    if (rr >= p.q_tokens * p.group) {
        c.state = 3;
        return c;
    }
    const int t = rr / p.group;
    c.len = seq_len - (p.q_tokens - 1 - t);
    const bool in_range = c.len >= 0 && c.len <= p.max_context_len && c.len <= p.blocks_per_seq * p.block_size;
    c.state = !in_range ? 2 : (c.len == 0 ? 1 : 0);
    if (c.state == 0) {
        const int64_t pages = (c.len + 15) / 16;
        const int64_t splits = (pages + p.pages_per_split - 1) / p.pages_per_split;
        c.splits = splits < 1 ? 1 : static_cast<int>(splits);
    }
    return c;
}

// Longest context among a tile's attending rows [first_rr, last_rr] (0 if
// none). Rows are token-major, row r attends seq_len - (T - 1 - r / G)
// tokens, and a row attends when that is in [1, cap] (chunk_row), so the
// tile's lengths are consecutive integers and the longest attending one is
// min(last row's, cap).
__device__ __forceinline__ int64_t tile_max_len(const DecodeParams& p, int64_t seq_len, int first_rr, int last_rr) {
    const int64_t cap = min(p.max_context_len, p.blocks_per_seq * p.block_size);
    const int64_t lo = seq_len - (p.q_tokens - 1 - first_rr / p.group);
    const int64_t hi = seq_len - (p.q_tokens - 1 - last_rr / p.group);
    if (hi < 1 || lo > cap) return 0;
    return min(hi, cap);
}

template <typename T, int D>
__global__ void __launch_bounds__(kChunkThreads, 3)
paged_chunk_mma_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                       const __grid_constant__ CUtensorMap vmap, int q_tiles) {
    using Shape = ChunkShape<D>;
    using Op = MmaOp<T>;
    constexpr int S = Shape::kStages;
    constexpr int KS = D / 16;   // k-steps of Q.K^T
    constexpr int NO = D / 8;    // n-tiles of the output

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t full[kChunkMaxStages];
    __shared__ __align__(8) uint64_t empty[kChunkMaxStages];
    __shared__ int s_ids[kChunkMaxPages];
    __shared__ int s_first_bad;   // first corrupted page of the split (relative), or n

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int tile = blockIdx.x % q_tiles;
    const int split = blockIdx.x / q_tiles;
    const int h = blockIdx.y;
    const int b = blockIdx.z;
    const int G = p.group;

    wait_for_prior_grid();
    allow_next_grid();
    const int64_t seq_len = p.context_lens ? load_index(p.context_lens, p.lens_i64, b) : p.uniform_len;
    // The tile's rows are token-major, so its last real row has its longest context.
    const int rows_total = p.q_tokens * G;
    const int last_rr = min(tile * kChunkRows + kChunkRows, rows_total) - 1;
    const int64_t max_len = tile_max_len(p, seq_len, tile * kChunkRows, last_rr);
    // Warps that hold rows of this tile; the others leave at once.
    const int active = min(kChunkWarps, (rows_total - tile * kChunkRows + 15) / 16);
    const int64_t pages_max = (max_len + 15) / 16;
    const int64_t page_begin = static_cast<int64_t>(split) * p.pages_per_split;
    const int64_t page_end = min(page_begin + p.pages_per_split, pages_max);
    const int n_pages = page_end > page_begin ? static_cast<int>(page_end - page_begin) : 0;  // <= kChunkMaxPages
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const uint32_t smem_base = smem_addr(smem);

    if (threadIdx.x == 0) {
        for (int st = 0; st < S; ++st) {
            mbar_init(smem_addr(&full[st]), 1);
            mbar_init(smem_addr(&empty[st]), active);
        }
    }
    // Warp 0 stages the split's page IDs and finds its first corrupted one
    // (never loaded: no row that reaches it survives).
    if (warp == 0) {
        int first_bad = n_pages;
        for (int i0 = 0; i0 < n_pages; i0 += 32) {
            const int i = i0 + lane;
            bool bad = false;
            if (i < n_pages) {
                const int64_t id = load_index(p.block_table, p.table_i64, b * p.table_stride + page_begin + i);
                bad = id < 0 || id >= p.num_blocks;
                s_ids[i] = bad ? 0 : static_cast<int>(id);
            }
            const unsigned mask = __ballot_sync(0xffffffffu, bad);
            if (mask) {
                if (lane == 0) report_bad_page_id();
                first_bad = i0 + __ffs(mask) - 1;
                break;
            }
        }
        if (lane == 0) s_first_bad = first_bad;
    }
    fence_mbar_init();
    __syncthreads();
    if (warp >= active) return;
    const int first_bad = s_first_bad;
    const int n_use = first_bad;

    // Thread 0 issues page j into stage j % S; `issued` counts its loads.
    const bool issuer = threadIdx.x == 0;
    int issued = 0;
    bool issue_failed = false;
    auto issue = [&](int j) {
        const uint32_t bar = smem_addr(&full[j % S]);
        const uint32_t dst = smem_base + (j % S) * Shape::kStageBytes;
        mbar_arrive_expect_tx(bar, Shape::kStageBytes);
        tma_load_5d(dst, &kmap, 0, 0, 0, h, s_ids[j], bar);
        tma_load_5d(dst + Shape::kTileBytes, &vmap, 0, 0, 0, h, s_ids[j], bar);
        issued = j + 1;
    };
    if (issuer) {
        for (int j = 0; j < S && j < n_use; ++j) issue(j);
    }

    // ---- rows row_a = warp*16 + lane/4 and row_b = row_a + 8 of the tile
    const int rr_a = tile * kChunkRows + warp * 16 + (lane >> 2);
    const int rr_b = rr_a + 8;
    const ChunkRow ca = chunk_row(p, b, rr_a, seq_len);
    const ChunkRow cb = chunk_row(p, b, rr_b, seq_len);
    // A row takes part in this split when its context reaches into it.
    const bool in_a = ca.state == 0 && split < ca.splits;
    const bool in_b = cb.state == 0 && split < cb.splits;
    // Token positions relative to the split's first token, clamped into int
    // range (-1: nothing of the split).
    const int64_t split_tok = page_begin * 16;
    auto rel = [&](int64_t pos) -> int {
        const int64_t d = pos - split_tok;
        return d < -1 ? -1 : (d > (1 << 30) ? (1 << 30) : static_cast<int>(d));
    };
    const int pos_a = in_a ? rel(ca.len - 1) : -1;   // last token the row attends
    const int pos_b = in_b ? rel(cb.len - 1) : -1;
    const int cta_pos = rel(max_len - 1);             // tokens after it hold no data for any row

    // Q rows as mma A fragments (rows the tile does not have read row 0 of head 0; masked).
    uint32_t qa[KS][4];
    {
        const int c2 = 2 * (lane & 3);
        const uint16_t* q = static_cast<const uint16_t*>(p.q);
        const int ra = ca.state == 3 ? 0 : rr_a, rb = cb.state == 3 ? 0 : rr_b;
        const uint16_t* qra = q + b * p.q_stride_seq + static_cast<int64_t>(h * G + ra % G) * p.q_stride_head +
                              static_cast<int64_t>(ra / G) * p.q_stride_token;
        const uint16_t* qrb = q + b * p.q_stride_seq + static_cast<int64_t>(h * G + rb % G) * p.q_stride_head +
                              static_cast<int64_t>(rb / G) * p.q_stride_token;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int d = ks * 16 + c2;
            qa[ks][0] = *reinterpret_cast<const uint32_t*>(qra + d);
            qa[ks][1] = *reinterpret_cast<const uint32_t*>(qrb + d);
            qa[ks][2] = *reinterpret_cast<const uint32_t*>(qra + d + 8);
            qa[ks][3] = *reinterpret_cast<const uint32_t*>(qrb + d + 8);
        }
    }
    float o[NO][4];
#pragma unroll
    for (int j = 0; j < NO; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.0f, l_b = 0.0f;
    bool failed = false;

    const int k_tok = (lane & 7) + ((lane >> 4) & 1) * 8;   // B = K: matrices (tok 0-7, d lo/hi), (tok 8-15, ...)
    const int k_hi = (lane >> 3) & 1;
    const int v_tok = (lane & 7) + ((lane >> 3) & 1) * 8;   // B = V via .trans: (tok 0-7 / 8-15) x d pair
    const int v_hi = lane >> 4;

    int i = 0;
    for (; i < n_use; ++i) {
        const int st = i % S;
        const bool ok = mbar_wait_bounded(smem_addr(&full[st]), (i / S) & 1);
        if (!__all_sync(0xffffffffu, ok)) {
            failed = true;
            break;
        }
        const uint32_t kt = smem_base + st * Shape::kStageBytes;
        const uint32_t vt = kt + Shape::kTileBytes;
        const int tok0 = i * 16;

        // S = Q K^T for the page's 16 tokens (two n-tiles of 8); even and odd
        // k-steps accumulate apart, so four mma chains are in flight.
        float s0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        float s2[4] = {0.0f, 0.0f, 0.0f, 0.0f}, s3[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            uint32_t kb[4];
            const int r = (ks >> 2) * 16 + k_tok;
            const int c = ((ks & 3) << 1) + k_hi;
            ldmatrix_x4(kb, kt + r * 128 + ((c ^ (r & 7)) << 4));
            if (ks & 1) {
                Op::run(s2, qa[ks], kb[0], kb[1]);
                Op::run(s3, qa[ks], kb[2], kb[3]);
            } else {
                Op::run(s0, qa[ks], kb[0], kb[1]);
                Op::run(s1, qa[ks], kb[2], kb[3]);
            }
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            s0[e] += s2[e];
            s1[e] += s3[e];
        }
        // Causal mask per row, then the online softmax (scores in the exp2 domain).
        const int j0 = tok0 + 2 * (lane & 3);
        float x[8];
        x[0] = j0 <= pos_a ? s0[0] * p.scale_log2 : -INFINITY;
        x[1] = j0 + 1 <= pos_a ? s0[1] * p.scale_log2 : -INFINITY;
        x[2] = j0 <= pos_b ? s0[2] * p.scale_log2 : -INFINITY;
        x[3] = j0 + 1 <= pos_b ? s0[3] * p.scale_log2 : -INFINITY;
        x[4] = j0 + 8 <= pos_a ? s1[0] * p.scale_log2 : -INFINITY;
        x[5] = j0 + 9 <= pos_a ? s1[1] * p.scale_log2 : -INFINITY;
        x[6] = j0 + 8 <= pos_b ? s1[2] * p.scale_log2 : -INFINITY;
        x[7] = j0 + 9 <= pos_b ? s1[3] * p.scale_log2 : -INFINITY;
        float mx_a = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[4], x[5]));
        float mx_b = fmaxf(fmaxf(x[2], x[3]), fmaxf(x[6], x[7]));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
        const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
        // A row with nothing attended yet keeps m = -inf: scale 1, weights 0.
        const float sc_a = mn_a == -INFINITY ? 1.0f : fast_exp2(m_a - mn_a);
        const float sc_b = mn_b == -INFINITY ? 1.0f : fast_exp2(m_b - mn_b);
        const float base_a = mn_a == -INFINITY ? 0.0f : mn_a;
        const float base_b = mn_b == -INFINITY ? 0.0f : mn_b;
        float pr[8];
        pr[0] = fast_exp2(x[0] - base_a);
        pr[1] = fast_exp2(x[1] - base_a);
        pr[2] = fast_exp2(x[2] - base_b);
        pr[3] = fast_exp2(x[3] - base_b);
        pr[4] = fast_exp2(x[4] - base_a);
        pr[5] = fast_exp2(x[5] - base_a);
        pr[6] = fast_exp2(x[6] - base_b);
        pr[7] = fast_exp2(x[7] - base_b);
        m_a = mn_a;
        m_b = mn_b;
        l_a = l_a * sc_a + (pr[0] + pr[1] + pr[4] + pr[5]);
        l_b = l_b * sc_b + (pr[2] + pr[3] + pr[6] + pr[7]);
#pragma unroll
        for (int j = 0; j < NO; ++j) {
            o[j][0] *= sc_a;
            o[j][1] *= sc_a;
            o[j][2] *= sc_b;
            o[j][3] *= sc_b;
        }
        // P as the A operand of P.V: the two S n-tiles are its k halves.
        uint32_t pa[4];
        pa[0] = Op::pack(pr[0], pr[1]);
        pa[1] = Op::pack(pr[2], pr[3]);
        pa[2] = Op::pack(pr[4], pr[5]);
        pa[3] = Op::pack(pr[6], pr[7]);
        // Tokens past every row's context may hold anything (NaN too): zero their
        // V entries in the fragments (P is 0 there, but 0 * NaN is NaN).
        const int valid = min(16, cta_pos + 1 - tok0);
        const int t_lo = 2 * (lane & 3);
        const uint32_t keep_b0 = (t_lo < valid ? 0x0000ffffu : 0u) | (t_lo + 1 < valid ? 0xffff0000u : 0u);
        const uint32_t keep_b1 = (t_lo + 8 < valid ? 0x0000ffffu : 0u) | (t_lo + 9 < valid ? 0xffff0000u : 0u);
#pragma unroll
        for (int jj = 0; jj < NO / 2; ++jj) {
            uint32_t vb[4];
            const int r = ((jj * 16) >> 6) * 16 + v_tok;
            const int c = (((jj * 16) & 63) >> 3) + v_hi;
            ldmatrix_x4_trans(vb, vt + r * 128 + ((c ^ (r & 7)) << 4));
            Op::run(o[2 * jj], pa, vb[0] & keep_b0, vb[1] & keep_b1);
            Op::run(o[2 * jj + 1], pa, vb[2] & keep_b0, vb[3] & keep_b1);
        }
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&empty[st])) : "memory");
        // Refill the stage of page i - 1 with page i - 1 + S once every warp released it.
        const int j = i - 1 + S;
        if (issuer && i >= 1 && j < n_use && !issue_failed) {
            if (mbar_wait_bounded(smem_addr(&empty[(i - 1) % S]), ((i - 1) / S) & 1)) {
                issue(j);
            } else {
                issue_failed = true;
                atomicOr(&g_device_status, kStatusWaitTimeout);
            }
        }
    }
    if (failed) {
        if (lane == 0) atomicOr(&g_device_status, kStatusWaitTimeout);
    }
    // The CTA (and its shared memory) lives until every load it issued has
    // landed, whatever the warps did (bounded waits).
    if (issuer) {
        for (int jj = issued > S ? issued - S : 0; jj < issued; ++jj)
            mbar_wait_bounded(smem_addr(&full[jj % S]), (jj / S) & 1);
    }

    // Row sums over the quad, then the results.
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
    l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
    const float nan = __int_as_float(0x7fffffff);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        const ChunkRow c = chunk_row(p, b, half ? rr_b : rr_a, seq_len);
        const int rr = half ? rr_b : rr_a;
        const bool in = half ? in_b : in_a;
        const float mrow = half ? m_b : m_a;
        const float lrow = half ? l_b : l_a;
        if (c.state == 3) continue;
        const int t = rr / G;
        const int hq = h * G + rr % G;
        const int64_t z = static_cast<int64_t>(b) * p.q_tokens + t;
        T* out = static_cast<T*>(p.out) + row_out_offset(p, z) + static_cast<int64_t>(hq) * p.out_stride_head;
        if (!in) {
            // Constant rows (empty: zeros; invalid: NaN) are written once, by split 0.
            if (c.state != 0 && split == 0) {
                const float value = c.state == 1 ? 0.0f : nan;
                for (int d = 2 * (lane & 3); d < D; d += 8) {
                    out[d] = from_float<T>(value);
                    out[d + 1] = from_float<T>(value);
                }
            }
            continue;
        }
        // A corrupted page inside this row's part of the split, or a wait that gave up: NaN.
        const int64_t row_end = min(page_begin + p.pages_per_split, (c.len + 15) / 16);
        const bool poisoned = failed || page_begin + first_bad < row_end;
        const float inv = 1.0f / lrow;
        if (c.splits == 1) {
#pragma unroll
            for (int j = 0; j < NO; ++j) {
                const int d = j * 8 + 2 * (lane & 3);
                out[d] = from_float<T>(poisoned ? nan : o[j][half * 2] * inv);
                out[d + 1] = from_float<T>(poisoned ? nan : o[j][half * 2 + 1] * inv);
            }
        } else {
            const int64_t row = (z * p.q_heads + hq) * p.max_splits + split;
#pragma unroll
            for (int j = 0; j < NO; ++j) {
                const int d = j * 8 + 2 * (lane & 3);
                p.part_o[row * D + d] = poisoned ? nan : o[j][half * 2] * inv;
                p.part_o[row * D + d + 1] = poisoned ? nan : o[j][half * 2 + 1] * inv;
            }
            if ((lane & 3) == 0) p.part_lse[row] = poisoned ? nan : mrow + log2f(lrow);
        }
    }
}

}  // namespace mv
