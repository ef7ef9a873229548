// Attention of a chunk of T new tokens per sequence over its pages on the
// 5th-generation tensor cores: 128 query rows per CTA, tcgen05.mma with the
// accumulators in tensor memory (TMEM), K/V pages staged by TMA.
//
// Query rows of one (sequence b, KV head h) are r = t * G + g (chunk token t,
// query head h*G + g); row r attends the first len - (T - 1 - t) tokens. A
// CTA owns 128 rows (one per TMEM lane) and one split of the pages, taken in
// groups of four pages (64 tokens):
//   S[128, 64]  = Q[128, D] . K_group^T     tcgen05.mma kind::f16 (N = 64), A = Q and B =
//                                           the group's four K pages in shared memory
//                                           (K-major, 128-byte swizzle: TMA lands each
//                                           64-dim half of a page at its rows), D in TMEM
//   softmax     one thread per row: tcgen05.ld of its S row, causal mask, running
//               max in the exp2 domain, P = 2^(s - m) packed to 16 bits and stored
//               back over S in TMEM (tcgen05.st)
//   O[128, D]  += P[128, 64] . V_group      tcgen05.mma with A = P from TMEM and B =
//                                           the V page tiles (MN-major, 128-byte swizzle)
// The running max is rescaled lazily: O (in TMEM) is multiplied only when a
// row's max grows by more than 2^8, so the sums stay exact in fp32 and the
// read-modify-write of O is rare.
//
// Warps: 0-3 softmax (warp w owns TMEM lanes 32w..32w+31), 4 issues the S
// MMAs (one thread) and owns the TMEM allocation, 7 issues the P.V MMAs (so a
// group's P.V never queues behind the next group's S), 5 and 6 issue the TMA loads of
// the K and the V pages into separate rings: a K page is released as soon as
// its S MMAs complete, so K runs a group or more ahead of the softmax, and V
// only has to arrive by its group's P.V. S is double-buffered (S of group
// i+1 is computed while group i's softmax runs); P aliases its group's S
// columns. Every wait is bounded (2 s): a wait that gives up sets the device
// status, stops the CTA's issuers, poisons the rows, and the CTA still
// drains its loads and MMAs before freeing TMEM.
//
// Results use the decode path's row format (output rows, or normalised
// partials + log2-sum-exp merged by the split merge), as the mma.sync tile
// kernel does.
#pragma once

#include "mv_device.cuh"
#include "paged_chunk_mma.cuh"

namespace mv {

constexpr int kUmmaRows = 128;
constexpr int kUmmaSoftmaxWarps = 4;
constexpr int kUmmaMmaWarp = 4;
constexpr int kUmmaKWarp = 5;
constexpr int kUmmaVWarp = 6;
constexpr int kUmmaPvWarp = 7;
constexpr int kUmmaThreads = 8 * 32;
constexpr int kUmmaGroupPages = 4;          // pages (of 16 tokens) per softmax group
constexpr int kUmmaTmemCols = 256;

template <int D>
struct UmmaShape {
    static constexpr int kStages = D == 64 ? 16 : 8;     // pages in each of the K and V rings
    static constexpr int kTileBytes = 16 * D * 2;        // one K (or V) page of one head
    static constexpr int kQBytes = kUmmaRows * D * 2;    // [D/64][128 rows][128 B]
    static constexpr int kRingBytes = kStages * kTileBytes;
    // K ring: [group slot][D / 64][64 tokens][128 B], the group's pages at rows 16 j.
    static constexpr int kKSlotBytes = (D / 64) * 64 * 128;
    static constexpr int kSmemBytes = kQBytes + 2 * kRingBytes + 1024;
    static constexpr int kOCol = 0;                      // O: columns [0, D)
    static constexpr int kSCol = D;                      // S buffers: [D + 64 b, D + 64 b + 64)
    static_assert(kSCol + 2 * 64 <= kUmmaTmemCols, "TMEM columns");
    static_assert(kStages % kUmmaGroupPages == 0, "whole groups in the ring");
};

// Shared-memory matrix descriptor of a 128-byte-swizzled tile (sm_100 format:
// start >> 4, leading and stride byte offsets >> 4, version 1, layout 2).
__device__ __forceinline__ uint64_t umma_sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFF) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32) | (static_cast<uint64_t>(1) << 46) |
           (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor of kind::f16 with fp32 accumulators: A/B format
// (0 fp16, 1 bf16), majors (0 K, 1 MN), N >> 3, M >> 4.
template <typename T>
__host__ __device__ constexpr uint32_t umma_idesc(int m, int n, int b_mn) {
    constexpr uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
    return (1u << 4) | (fmt << 7) | (fmt << 10) | (static_cast<uint32_t>(b_mn) << 16) |
           (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
        "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

template <typename T, int D>
__global__ void __launch_bounds__(kUmmaThreads, 1)
paged_chunk_umma_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, int q_tiles) {
    using Shape = UmmaShape<D>;
    using Op = MmaOp<T>;
    constexpr int NS = Shape::kStages;
    constexpr int KS = D / 16;   // k-steps of Q.K^T

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t k_full[NS];
    __shared__ __align__(8) uint64_t k_empty[NS];
    __shared__ __align__(8) uint64_t v_full[NS];
    __shared__ __align__(8) uint64_t v_empty[NS];
    __shared__ __align__(8) uint64_t s_full[2];
    __shared__ __align__(8) uint64_t p_ready[2];
    __shared__ __align__(8) uint64_t o_done;
    __shared__ __align__(8) uint64_t p_free[2];
    __shared__ __align__(8) uint64_t drained;
    __shared__ int s_ids[kChunkMaxPages];      // page IDs of the K producer
    __shared__ int s_vids[kChunkMaxPages];     // the same, loaded by the V producer
    __shared__ int s_first_bad;
    __shared__ uint32_t s_tmem;
    __shared__ volatile int s_failed;

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
    const int rows_total = p.q_tokens * G;
    const int last_rr = min(tile * kUmmaRows + kUmmaRows, rows_total) - 1;
    const int64_t max_len = tile_max_len(p, seq_len, tile * kUmmaRows, last_rr);
    const int64_t pages_max = (max_len + 15) / 16;
    const int64_t page_begin = static_cast<int64_t>(split) * p.pages_per_split;
    const int64_t page_end = min(page_begin + p.pages_per_split, pages_max);
    const int n_pages = page_end > page_begin ? static_cast<int>(page_end - page_begin) : 0;  // <= kChunkMaxPages
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint8_t* q_smem = smem;
    const uint32_t q_base = smem_addr(q_smem);
    const uint32_t k_ring = q_base + Shape::kQBytes;
    const uint32_t v_ring = k_ring + Shape::kRingBytes;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(smem_addr(&s_full[i]), 1);
            mbar_init(smem_addr(&p_ready[i]), kUmmaSoftmaxWarps);
            mbar_init(smem_addr(&p_free[i]), 1);
        }
        mbar_init(smem_addr(&o_done), 1);
        mbar_init(smem_addr(&drained), 2);   // one final commit per MMA issuer
        s_failed = 0;
    }
    if (warp == kUmmaMmaWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                     "r"(kUmmaTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    // Producers (warp 5: K pages, warp 6: V pages) start before the CTA-wide
    // barrier: each initialises its own ring's barriers, loads the split's
    // page IDs itself and issues the ring's first pages, so those loads
    // overlap the Q rows' loads below.
    int first_bad = n_pages;   // the split's first corrupted page (never loaded)
    int prod_next = 0;         // producer lanes: next page to issue
    if (warp == kUmmaKWarp || warp == kUmmaVWarp) {
        const bool is_k = warp == kUmmaKWarp;
        uint64_t* full = is_k ? k_full : v_full;
        uint64_t* empty = is_k ? k_empty : v_empty;
        int* ids = is_k ? s_ids : s_vids;
        if (lane == 0) {
            for (int st = 0; st < NS; ++st) {
                mbar_init(smem_addr(&full[st]), 1);
                mbar_init(smem_addr(&empty[st]), 1);
            }
            fence_mbar_init();
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(is_k ? &kmap : &vmap))
                         : "memory");
        }
        for (int i0 = 0; i0 < n_pages; i0 += 32) {
            const int i = i0 + lane;
            bool bad = false;
            if (i < n_pages) {
                const int64_t id = load_index(p.block_table, p.table_i64, b * p.table_stride + page_begin + i);
                bad = id < 0 || id >= p.num_blocks;
                ids[i] = bad ? 0 : static_cast<int>(id);
            }
            const unsigned mask = __ballot_sync(0xffffffffu, bad);
            if (mask) {
                if (is_k && lane == 0) report_bad_page_id();
                first_bad = i0 + __ffs(mask) - 1;
                break;
            }
        }
        if (is_k && lane == 0) s_first_bad = first_bad;
        __syncwarp();
        // The ring's first pages need no free stage: one per lane, four lanes
        // issuing a group's four pages together.
        prod_next = lane;
        if (lane < kUmmaGroupPages) {
            const CUtensorMap* map = is_k ? &kmap : &vmap;
            const uint32_t ring = is_k ? k_ring : v_ring;
            for (; prod_next < first_bad && prod_next < NS; prod_next += kUmmaGroupPages) {
                const int j = prod_next;
                const uint32_t bar = smem_addr(&full[j]);
                mbar_arrive_expect_tx(bar, Shape::kTileBytes);
                if (is_k) {
                    const uint32_t slot = ring + (j / kUmmaGroupPages) * Shape::kKSlotBytes + (j % kUmmaGroupPages) * 2048;
#pragma unroll
                    for (int a = 0; a < D / 64; ++a) tma_load_5d(slot + a * 8192, map, 0, 0, a, h, ids[j], bar);
                } else {
                    tma_load_5d(ring + j * Shape::kTileBytes, map, 0, 0, 0, h, ids[j], bar);
                }
            }
        }
    }
    // Q rows into shared memory in the MMA's K-major 128-byte-swizzled layout:
    // element (row, d) at [d / 64][row][16-byte chunk ((d % 64) / 8) ^ (row % 8)].
    if (warp < kUmmaSoftmaxWarps) {
        // Lanes of a row group read one row's 16-byte pieces; every load of the
        // thread is issued before the first store (one round of latency).
        constexpr int kChunks = D / 8;                                   // 16-byte chunks per row
        constexpr int kPer = kUmmaRows * kChunks / (kUmmaSoftmaxWarps * 32);
        const uint8_t* q = static_cast<const uint8_t*>(p.q);
        uint4 v[kPer];
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int idx = threadIdx.x + u * kUmmaSoftmaxWarps * 32;
            const int r = idx / kChunks;
            const int c = idx - r * kChunks;
            const int rr = tile * kUmmaRows + r;
            v[u] = make_uint4(0u, 0u, 0u, 0u);
            if (rr < rows_total) {
                const int64_t off = (b * p.q_stride_seq + static_cast<int64_t>(h * G + rr % G) * p.q_stride_head +
                                     static_cast<int64_t>(rr / G) * p.q_stride_token) * 2 + c * 16;
                v[u] = __ldg(reinterpret_cast<const uint4*>(q + off));
            }
        }
#pragma unroll
        for (int u = 0; u < kPer; ++u) {
            const int idx = threadIdx.x + u * kUmmaSoftmaxWarps * 32;
            const int r = idx / kChunks;
            const int c = idx - r * kChunks;
            *reinterpret_cast<uint4*>(q_smem + (c >> 3) * (kUmmaRows * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4)) =
                v[u];
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    fence_mbar_init();
    tmem_fence_before();
    __syncthreads();
    tmem_fence_after();
    const uint32_t tmem = s_tmem;
    const int n_use = s_first_bad;
    const int n_groups = (n_use + kUmmaGroupPages - 1) / kUmmaGroupPages;

    if (warp == kUmmaKWarp || warp == kUmmaVWarp) {
        // Producers: page j's K (warp 5) or V (warp 6) tile into stage j % NS of
        // its ring once the MMAs that read the stage's previous page finished
        // (the empty barriers are committed by the MMA thread).
        const bool is_k = warp == kUmmaKWarp;
        uint64_t* full = is_k ? k_full : v_full;
        uint64_t* empty = is_k ? k_empty : v_empty;
        const CUtensorMap* map = is_k ? &kmap : &vmap;
        const uint32_t ring = is_k ? k_ring : v_ring;
        const int* ids = is_k ? s_ids : s_vids;
        // Four lanes issue the four pages of a group together (one TMA
        // instruction for all four), each waiting for its own stage; the
        // ring's first pages went out before the CTA barrier.
        if (lane < kUmmaGroupPages) {
            int last = prod_next - kUmmaGroupPages;   // this lane's last page issued
            for (int j = prod_next; j < n_use; j += kUmmaGroupPages) {
                const int st = j % NS;
                if (j >= NS && !mbar_wait_bounded(smem_addr(&empty[st]), ((j / NS) - 1) & 1)) {
                    s_failed = 1;
                    atomicOr(&g_device_status, kStatusWaitTimeout);
                    break;
                }
                if (s_failed) break;
                const uint32_t bar = smem_addr(&full[st]);
                mbar_arrive_expect_tx(bar, Shape::kTileBytes);
                if (is_k) {
                    // Each 64-dim half of the page at rows 16 (j % 4) of its group slot.
                    const uint32_t slot = ring + (st / kUmmaGroupPages) * Shape::kKSlotBytes + (st % kUmmaGroupPages) * 2048;
#pragma unroll
                    for (int a = 0; a < D / 64; ++a) tma_load_5d(slot + a * 8192, map, 0, 0, a, h, ids[j], bar);
                } else {
                    tma_load_5d(ring + st * Shape::kTileBytes, map, 0, 0, 0, h, ids[j], bar);
                }
                last = j;
            }
            // Every load issued lands before the CTA can exit: only this lane's
            // last NS / 4 pages can still be in flight.
            for (int j = last; j >= 0 && j > last - NS; j -= kUmmaGroupPages)
                mbar_wait_bounded(smem_addr(&full[j % NS]), (j / NS) & 1);
        }
        __syncwarp();
    } else if (warp == kUmmaMmaWarp || warp == kUmmaPvWarp) {
        // MMA issuers, one thread each. Warp 4: S of group g into buffer g % 2 once
        // the P.V of group g - 2 (which read P from that buffer) completed, so S
        // runs up to two groups ahead of the softmax. Warp 7: P.V of group g once
        // the softmax stored its P.
        if (lane == 0) {
            bool ok = true;
            if (warp == kUmmaMmaWarp) {
                const uint32_t s_idesc = umma_idesc<T>(kUmmaRows, kUmmaGroupPages * 16, 0);
                for (int g = 0; ok && g < n_groups; ++g) {
                    if (g >= 2 && !mbar_wait_bounded(smem_addr(&p_free[g & 1]), ((g >> 1) - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    for (int jj = 0; jj < kUmmaGroupPages && ok; ++jj) {
                        const int j = g * kUmmaGroupPages + jj;
                        if (j >= n_use) break;
                        ok = mbar_wait_bounded(smem_addr(&k_full[j % NS]), (j / NS) & 1);
                    }
                    if (!ok) break;
                    tmem_fence_after();
                    // All 64 rows of the group slot are read; rows of pages past
                    // n_use hold older pages and their scores are masked.
                    const uint32_t s_col = tmem + Shape::kSCol + (g & 1) * 64;
                    const uint32_t k_slot = k_ring + ((g * kUmmaGroupPages) % NS / kUmmaGroupPages) * Shape::kKSlotBytes;
#pragma unroll
                    for (int ks = 0; ks < KS; ++ks) {
                        const uint64_t a = umma_sw128_desc(q_base + (ks >> 2) * (kUmmaRows * 128) + (ks & 3) * 32, 16, 1024);
                        const uint64_t bd = umma_sw128_desc(k_slot + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024);
                        umma_ss(s_col, a, bd, s_idesc, ks > 0);
                    }
                    umma_commit(smem_addr(&s_full[g & 1]));
                    // The group's K pages are free once these MMAs complete.
                    for (int jj = 0; jj < kUmmaGroupPages; ++jj) {
                        const int j = g * kUmmaGroupPages + jj;
                        if (j >= n_use) break;
                        umma_commit(smem_addr(&k_empty[j % NS]));
                    }
                }
            } else {
                const uint32_t o_idesc = umma_idesc<T>(kUmmaRows, D, 1);
                for (int g = 0; ok && g < n_groups; ++g) {
                    if (!mbar_wait_bounded(smem_addr(&p_ready[g & 1]), (g >> 1) & 1)) {
                        ok = false;
                        break;
                    }
                    tmem_fence_after();
                    const uint32_t p_col = tmem + Shape::kSCol + (g & 1) * 64;
                    for (int jj = 0; jj < kUmmaGroupPages && ok; ++jj) {
                        const int j = g * kUmmaGroupPages + jj;
                        if (j >= n_use) break;
                        if (!mbar_wait_bounded(smem_addr(&v_full[j % NS]), (j / NS) & 1)) {
                            ok = false;
                            break;
                        }
                        const uint32_t v_tile = v_ring + (j % NS) * Shape::kTileBytes;
                        umma_ts(tmem + Shape::kOCol, p_col + jj * 8, umma_sw128_desc(v_tile, 2048, 1024), o_idesc,
                                g > 0 || jj > 0);
                    }
                    if (!ok) break;
                    umma_commit(smem_addr(&o_done));
                    umma_commit(smem_addr(&p_free[g & 1]));
                    for (int jj = 0; jj < kUmmaGroupPages; ++jj) {
                        const int j = g * kUmmaGroupPages + jj;
                        if (j >= n_use) break;
                        umma_commit(smem_addr(&v_empty[j % NS]));
                    }
                }
            }
            if (!ok) {
                s_failed = 1;
                atomicOr(&g_device_status, kStatusWaitTimeout);
            }
            // Every MMA issued completes before its results are read, and before
            // TMEM (and the stages) can be freed.
            umma_commit(smem_addr(&drained));
            mbar_wait_bounded(smem_addr(&drained), 0);
        }
        __syncwarp();
    } else {
        // ---- softmax: thread = query row rr of the tile, TMEM lane threadIdx.x.
        // tcgen05.ld/st are warp-collective: every lane runs them, and every
        // wait is made warp-uniform before anything depends on it.
        const int rr = tile * kUmmaRows + threadIdx.x;
        const ChunkRow c = chunk_row(p, b, rr, seq_len);
        const bool in = c.state == 0 && split < c.splits;
        const int64_t split_tok = page_begin * 16;
        auto rel = [&](int64_t pos) -> int {
            const int64_t d = pos - split_tok;
            return d < -1 ? -1 : (d > (1 << 30) ? (1 << 30) : static_cast<int>(d));
        };
        const int pos = in ? rel(c.len - 1) : -1;     // last token the row attends, split-relative
        const int cta_pos = rel(max_len - 1);          // tokens after it hold no data for any row
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
        float m_run = -INFINITY, l_run = 0.0f;
        bool failed = false;
        for (int g = 0; g < n_groups; ++g) {
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_addr(&s_full[g & 1]), (g >> 1) & 1))) {
                failed = true;
                break;
            }
            tmem_fence_after();
            float s[64];
            const uint32_t s_col = lane_base + Shape::kSCol + (g & 1) * 64;
            tmem_ld16(s_col, s);
            tmem_ld16(s_col + 16, s + 16);
            tmem_ld16(s_col + 32, s + 32);
            tmem_ld16(s_col + 48, s + 48);
            tmem_wait_ld();
            const int tok0 = g * kUmmaGroupPages * 16;
            const int avail = min(kUmmaGroupPages * 16, (n_use - g * kUmmaGroupPages) * 16);
            // A group inside every row's causal prefix (all of it but the
            // diagonal and the split's last pages) needs no mask, and with a
            // positive scale the max of the raw scores gives the scaled max:
            // the scale is then folded into the exponent's FFMA below.
            const bool unmasked = p.scale_log2 > 0.0f && avail == kUmmaGroupPages * 16 &&
                                  __all_sync(0xffffffffu, tok0 + kUmmaGroupPages * 16 - 1 <= pos);
            float gmax = -INFINITY;
            if (unmasked) {
#pragma unroll
                for (int i = 0; i < 64; ++i) gmax = fmaxf(gmax, s[i]);
                gmax *= p.scale_log2;
            } else {
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    s[i] = (i < avail && tok0 + i <= pos) ? s[i] * p.scale_log2 : -INFINITY;
                    gmax = fmaxf(gmax, s[i]);
                }
            }
            const float m_new = fmaxf(m_run, gmax);
            const bool grow = m_run != -INFINITY && m_new > m_run + 8.0f;
            if (__any_sync(0xffffffffu, grow)) {
                // O is rescaled only after the previous group's P.V finished
                // (P of group g may be written without it: S of group g went
                // into its buffer after the P.V of group g - 2 completed).
                if (g >= 1 &&
                    !__all_sync(0xffffffffu, mbar_wait_bounded(smem_addr(&o_done), (g - 1) & 1))) {
                    failed = true;
                    break;
                }
                tmem_fence_after();
                const float f = grow ? fast_exp2(m_run - m_new) : 1.0f;
#pragma unroll 1
                for (int col = 0; col < D; col += 16) {
                    float o[16];
                    tmem_ld16(lane_base + Shape::kOCol + col, o);
                    tmem_wait_ld();
                    uint32_t w[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) w[i] = __float_as_uint(o[i] * f);
                    tmem_st16(lane_base + Shape::kOCol + col, w);
                }
                l_run *= f;
            }
            if (grow || m_run == -INFINITY) m_run = m_new;
            const float base = m_run == -INFINITY ? 0.0f : m_run;
            uint32_t pk[32];
            float sum = 0.0f;
            if (unmasked) {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float p0 = fast_exp2(fmaf(s[2 * i], p.scale_log2, -base));
                    const float p1 = fast_exp2(fmaf(s[2 * i + 1], p.scale_log2, -base));
                    sum += p0 + p1;
                    pk[i] = Op::pack(p0, p1);
                }
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) {
                    const float p0 = fast_exp2(s[2 * i] - base);
                    const float p1 = fast_exp2(s[2 * i + 1] - base);
                    sum += p0 + p1;
                    pk[i] = Op::pack(p0, p1);
                }
            }
            l_run += sum;
            tmem_st16(s_col, pk);
            tmem_st16(s_col + 16, pk + 16);
            // Tokens past every row's context may hold anything (NaN too): zero
            // their V rows in the last page (P is 0 there, but 0 * NaN is NaN).
            if (warp == 0) {
                const int last = cta_pos >> 4;   // split-relative page holding the last token
                const int valid = cta_pos + 1 - last * 16;
                if (last >= g * kUmmaGroupPages && last < (g + 1) * kUmmaGroupPages && last < n_use && valid < 16 &&
                    __all_sync(0xffffffffu, mbar_wait_bounded(smem_addr(&v_full[last % NS]), (last / NS) & 1))) {
                    uint8_t* v_tile = smem + Shape::kQBytes + Shape::kRingBytes + (last % NS) * Shape::kTileBytes;
                    constexpr int kRowChunks = D / 8;
                    for (int idx = lane; idx < 16 * kRowChunks; idx += 32) {
                        const int row = idx / kRowChunks;
                        const int ch = idx - row * kRowChunks;
                        if (row >= valid)
                            *reinterpret_cast<uint4*>(v_tile + (ch >> 3) * 2048 + row * 128 +
                                                      (((ch & 7) ^ (row & 7)) << 4)) = make_uint4(0u, 0u, 0u, 0u);
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                }
            }
            tmem_wait_st();
            tmem_fence_before();
            __syncwarp();
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&p_ready[g & 1]))
                                        : "memory");
        }
        // Every MMA done (the issuer's final commit: a one-phase barrier, so
        // waiting on it needs no phase tracking), then this row's result.
        if (!failed && n_groups > 0 &&
            !__all_sync(0xffffffffu, mbar_wait_bounded(smem_addr(&drained), 0)))
            failed = true;
        if (failed || s_failed) {
            failed = true;
            if (lane == 0) atomicOr(&g_device_status, kStatusWaitTimeout);
        }
        tmem_fence_after();
        const float nan = __int_as_float(0x7fffffff);
        const int t = rr / G;
        const int hq = h * G + rr % G;
        const int64_t z = static_cast<int64_t>(b) * p.q_tokens + t;
        const int64_t row_end = min(page_begin + p.pages_per_split, (c.len + 15) / 16);
        const bool poisoned = failed || page_begin + n_use < row_end;
        const int64_t prow = (z * p.q_heads + hq) * p.max_splits + split;
        // This row's destination: 1 output (a result, or the constant of an empty
        // or invalid row, written by split 0), 2 a partial of the split merge.
        const bool constant = c.state != 3 && !in && c.state != 0 && split == 0;
        const int kind = (in && c.splits > 1) ? 2 : ((in || constant) ? 1 : 0);
        const float inv = poisoned ? nan : 1.0f / l_run;
        const float cval = c.state == 1 ? 0.0f : nan;   // a constant row's value (TMEM not read)
        if (kind == 2 && !poisoned) p.part_lse[prow] = m_run + log2f(l_run);
        if (kind == 2 && poisoned) p.part_lse[prow] = nan;
        const uintptr_t dest = kind == 1 ? reinterpret_cast<uintptr_t>(static_cast<T*>(p.out) + row_out_offset(p, z) +
                                                                        static_cast<int64_t>(hq) * p.out_stride_head)
                                         : reinterpret_cast<uintptr_t>(p.part_o + prow * D);
        // The warp's 32 rows go out through its quarter of the (now unused) Q
        // shared memory, D/2 columns at a time as fp32 (16-byte pieces swizzled
        // by row), then row by row with the lanes along the row: coalesced.
        float* stage = reinterpret_cast<float*>(q_smem + warp * (32 * (D / 2) * 4));
        constexpr int kHalf = D / 2;
        const bool out_pairs = ((reinterpret_cast<uintptr_t>(p.out) | static_cast<uintptr_t>(
                                   (p.out_stride_seq | p.out_stride_token | p.out_stride_head) * sizeof(T))) & 3) == 0;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
#pragma unroll 1
            for (int col = 0; col < kHalf; col += 16) {
                float o[16];
                tmem_ld16(lane_base + Shape::kOCol + half * kHalf + col, o);   // warp-collective
                tmem_wait_ld();
#pragma unroll
                for (int q4 = 0; q4 < 4; ++q4) {
                    const int chunk = (col >> 2) + q4;                         // 16-byte piece of the row
                    const float4 v = constant ? make_float4(cval, cval, cval, cval)
                                              : make_float4(o[4 * q4] * inv, o[4 * q4 + 1] * inv,
                                                            o[4 * q4 + 2] * inv, o[4 * q4 + 3] * inv);
                    *reinterpret_cast<float4*>(stage + lane * kHalf + ((chunk ^ (lane & 7)) << 2)) = v;
                }
            }
            __syncwarp();
            for (int i = 0; i < 32; ++i) {
                const int k = __shfl_sync(0xffffffffu, kind, i);
                const uint64_t d = __shfl_sync(0xffffffffu, static_cast<unsigned long long>(dest), i);
                if (k == 0) continue;
                for (int e = 2 * lane; e < kHalf; e += 64) {   // a pair of columns per lane
                    const float2 v = *reinterpret_cast<const float2*>(stage + i * kHalf + ((((e >> 2) ^ (i & 7)) << 2) | (e & 3)));
                    const int cidx = half * kHalf + e;
                    if (k == 2) {
                        *reinterpret_cast<float2*>(reinterpret_cast<float*>(d) + cidx) = v;
                    } else if (out_pairs) {
                        *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(d) + cidx) = Op::pack(v.x, v.y);
                    } else {
                        reinterpret_cast<T*>(d)[cidx] = from_float<T>(v.x);
                        reinterpret_cast<T*>(d)[cidx + 1] = from_float<T>(v.y);
                    }
                }
            }
            __syncwarp();
        }
    }
    // Free TMEM once every warp is done with it (the MMA thread's last
    // commit was waited on by the softmax warps, or nothing was issued).
    tmem_fence_before();
    __syncthreads();
    if (warp == kUmmaMmaWarp) {
        tmem_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kUmmaTmemCols));
    }
}

}  // namespace mv
