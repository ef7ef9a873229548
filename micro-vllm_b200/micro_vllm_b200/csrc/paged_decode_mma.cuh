// Paged GQA decode on sm_100a: TMA page staging + tensor-core (mma.sync) tiles.
//
// One CTA owns (split, KV head h, sequence b): a run of pages_per_split pages
// of one sequence. Every query head of h's GQA group shares each K/V page
// read, so K/V bytes cross HBM once (the reference kernel re-reads them once
// per query head: online_attention.cuh:112-115).
//
// Inside the CTA each warp owns every NWARPS-th page of the run and runs its
// own STAGES-deep TMA ring: one elected lane issues two 5-D tiled bulk tensor
// loads per page (the K page and the V page of head h, each block_size x D,
// 128-byte swizzled) that complete on the stage's mbarrier; the warp waits,
// computes, and refills the stage. Page IDs for the warp's whole run are read
// once, coalesced, one per lane, validated, and broadcast by shuffle.
//
// Per 16-token page (block_size 16 = the mma M dimension):
//   S^T[16 tok, 8 q] = K_page[16 x D] . Q^T         mma m16n8k16, A = K via ldmatrix
//   online softmax on the fragment (exp2 domain, quad shuffles for the max)
//   P^T fragment from S's accumulator by movmatrix.trans (no shared memory)
//   O^T[D, 8 q] += V_page^T[D x 16 tok] . P^T       mma m16n8k16, A = V via ldmatrix.trans
// The GQA group (<= 8 per n-tile) is the mma N dimension, so a group of 7
// wastes one column of eight; D is the M dimension of the P.V product.
//
// Warps merge through shared memory at the end; a CTA that covers the whole
// sequence writes the final output, otherwise a normalised partial and its
// log2-sum-exp for the merge kernel.
#pragma once

#include "mv_device.cuh"

namespace mv {

template <int D, int NT, int NWARPS, int STAGES>
struct MmaDecodeShape {
    static constexpr int kBlock = 16;                      // tokens per page
    static constexpr int kTileBytes = kBlock * D * 2;      // one K (or V) page of one head
    static constexpr int kStageBytes = 2 * kTileBytes;
    static constexpr int kWarpBytes = STAGES * kStageBytes;
    static constexpr int kSmemBytes = NWARPS * kWarpBytes + 1024;  // + 1 KiB for alignment
    static constexpr int kQRows = 8 * NT;
    static constexpr int kRedStride = D + 4;
    static constexpr int kRedBytes = (kQRows * kRedStride + 2 * kQRows) * 4;
    static constexpr int kMaxPagesPerSplit = 32 * NWARPS;  // one page ID per lane per warp
    static_assert(D % 64 == 0, "pages are staged as 64-column (128-byte) swizzled boxes");
    static_assert(kRedBytes <= kWarpBytes, "warp merge buffer must fit the warp's stages");
};

template <typename T, int D, int NT, int NWARPS, int STAGES>
__global__ void __launch_bounds__(NWARPS * 32)
paged_decode_mma_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap) {
    using Shape = MmaDecodeShape<D, NT, NWARPS, STAGES>;
    using Op = MmaOp<T>;
    constexpr int KS = D / 16;  // k-steps of S = K q, and m-tiles of O^T = V^T P^T

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[NWARPS][STAGES];
    __shared__ int cta_bad;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int split = blockIdx.x;
    const int h = blockIdx.y;
    const int b = blockIdx.z;

    const SeqSplit seq = seq_split(p, b);
    if (split >= seq.splits) return;
    if (seq.state != 0) {
        write_group_constant<T>(p, b, h, seq.state == 1 ? 0.0f : __int_as_float(0x7fffffff));
        return;
    }
    const bool single = seq.splits == 1;

    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    const int64_t page_begin = static_cast<int64_t>(split) * p.pages_per_split;
    const int64_t page_end_raw = page_begin + p.pages_per_split;
    const int cta_pages =
        static_cast<int>((page_end_raw < seq.pages ? page_end_raw : seq.pages) - page_begin);
    const int n_my = warp < cta_pages ? (cta_pages - warp + NWARPS - 1) / NWARPS : 0;

    // Page IDs of this warp's pages: lane i holds page warp + i * NWARPS of the run.
    long long my_id = 0;
    bool bad = false;
    if (lane < n_my) {
        my_id = load_index(p.block_table, p.table_i64,
                           b * p.table_stride + page_begin + warp + lane * NWARPS);
        bad = my_id < 0 || my_id >= p.num_blocks;
    }
    if (threadIdx.x == 0) cta_bad = 0;
    const uint32_t bar0 = smem_addr(&bars[warp][0]);
    if (lane == 0) {
#pragma unroll
        for (int st = 0; st < STAGES; ++st) mbar_init(bar0 + 8 * st, 1);
    }
    fence_mbar_init();
    __syncthreads();
    if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(&cta_bad, 1);
    __syncthreads();
    if (cta_bad) {
        // A corrupted table entry: never read that page, poison the group.
        if (single) write_group_constant<T>(p, b, h, __int_as_float(0x7fffffff));
        else write_group_partial_nan(p, b, h, split);
        return;
    }

    uint8_t* wsm = smem + warp * Shape::kWarpBytes;
    const uint32_t wsm_addr = smem_addr(wsm);

    // Prologue: fill the ring.
    const int prologue = n_my < STAGES ? n_my : STAGES;
    for (int i = 0; i < prologue; ++i) {
        const long long id = __shfl_sync(0xffffffffu, my_id, i);
        if (lane == 0) {
            const uint32_t bar = bar0 + 8 * i;
            const uint32_t dst = wsm_addr + i * Shape::kStageBytes;
            mbar_arrive_expect_tx(bar, Shape::kStageBytes);
            tma_load_5d(dst, &kmap, 0, 0, 0, h, static_cast<int>(id), bar);
            tma_load_5d(dst + Shape::kTileBytes, &vmap, 0, 0, 0, h, static_cast<int>(id), bar);
        }
    }

    // Q as the B operand of S^T = K Q^T: lane holds q[g][16 ks + 2(lane%4) + {0,1,8,9}].
    uint32_t qf[KS][NT][2];
    {
        const uint16_t* qbase = static_cast<const uint16_t*>(p.q) + b * p.q_stride_seq;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int g = nt * 8 + (lane >> 2);
            const bool has = g < p.group;
            const uint16_t* qrow =
                qbase + static_cast<int64_t>(h * p.group + (has ? g : 0)) * p.q_stride_head;
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                const int d0 = ks * 16 + 2 * (lane & 3);
                qf[ks][nt][0] = has ? (static_cast<uint32_t>(qrow[d0]) |
                                       (static_cast<uint32_t>(qrow[d0 + 1]) << 16))
                                    : 0u;
                qf[ks][nt][1] = has ? (static_cast<uint32_t>(qrow[d0 + 8]) |
                                       (static_cast<uint32_t>(qrow[d0 + 9]) << 16))
                                    : 0u;
            }
        }
    }

    float m_run[NT][2];
    float l_run[NT][2];
    float o[KS][NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        m_run[nt][0] = m_run[nt][1] = -INFINITY;
        l_run[nt][0] = l_run[nt][1] = 0.0f;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.0f;
    }

    // Lane-constant parts of the ldmatrix row addresses (see the file comment).
    const int k_slot = (lane & 7) + ((lane >> 3) & 1) * 8;  // A = K: matrices (rows, cols) 00,10,01,11
    const int k_chunk = lane >> 4;
    const int v_tok = (lane & 7) + ((lane >> 4) & 1) * 8;   // A = V^T via .trans
    const int v_chunk = (lane >> 3) & 1;
    const int row0 = lane >> 2;                             // token of accumulator rows c0/c1

    bool failed = false;
    int i = 0;
    for (; i < n_my; ++i) {
        const int st = i % STAGES;
        const uint32_t parity = (i / STAGES) & 1;
        const bool ok = mbar_wait_bounded(bar0 + 8 * st, parity);
        if (!__all_sync(0xffffffffu, ok)) {
            failed = true;
            break;
        }
        const uint32_t kt = wsm_addr + st * Shape::kStageBytes;
        const uint32_t vt = kt + Shape::kTileBytes;
        const int64_t page = page_begin + warp + static_cast<int64_t>(i) * NWARPS;
        const int64_t left = seq.len - page * 16;
        const int valid = left < 16 ? static_cast<int>(left) : 16;
        if (valid < 16) {
            // Slots past the context in the last page may hold anything (NaN included);
            // P is 0 there, but 0 * NaN is NaN, so clear those V rows before P.V.
            uint8_t* vgen = wsm + st * Shape::kStageBytes + Shape::kTileBytes;
            const int rows = 16 - valid;
            for (int idx = lane; idx < (D / 64) * rows * 8; idx += 32) {
                const int chunk = idx & 7;
                const int rr = idx >> 3;
                const int half = rr / rows;
                const int slot = valid + (rr - half * rows);
                *reinterpret_cast<uint4*>(vgen + (half * 16 + slot) * 128 + chunk * 16) =
                    make_uint4(0u, 0u, 0u, 0u);
            }
            __syncwarp();
        }

        float sc[NT][4];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int r = (ks >> 2) * 16 + k_slot;
            const int c = ((ks & 3) << 1) + k_chunk;
            uint32_t a[4];
            ldmatrix_x4(a, kt + r * 128 + ((c ^ (r & 7)) << 4));
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) Op::run(sc[nt], a, qf[ks][nt][0], qf[ks][nt][1]);
        }

        const bool v0 = row0 < valid;
        const bool v1 = row0 + 8 < valid;
        uint32_t pb[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const float x0 = v0 ? sc[nt][0] * p.scale_log2 : -INFINITY;
            const float x1 = v0 ? sc[nt][1] * p.scale_log2 : -INFINITY;
            const float x2 = v1 ? sc[nt][2] * p.scale_log2 : -INFINITY;
            const float x3 = v1 ? sc[nt][3] * p.scale_log2 : -INFINITY;
            float mx0 = fmaxf(x0, x2);
            float mx1 = fmaxf(x1, x3);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float mn0 = fmaxf(m_run[nt][0], mx0);
            const float mn1 = fmaxf(m_run[nt][1], mx1);
            const float a0 = fast_exp2(m_run[nt][0] - mn0);
            const float a1 = fast_exp2(m_run[nt][1] - mn1);
            m_run[nt][0] = mn0;
            m_run[nt][1] = mn1;
            const float p0 = fast_exp2(x0 - mn0);
            const float p1 = fast_exp2(x1 - mn1);
            const float p2 = fast_exp2(x2 - mn0);
            const float p3 = fast_exp2(x3 - mn1);
            l_run[nt][0] = l_run[nt][0] * a0 + (p0 + p2);
            l_run[nt][1] = l_run[nt][1] * a1 + (p1 + p3);
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) {
                o[mt][nt][0] *= a0;
                o[mt][nt][1] *= a1;
                o[mt][nt][2] *= a0;
                o[mt][nt][3] *= a1;
            }
            pb[nt][0] = movmatrix_trans(Op::pack(p0, p1));
            pb[nt][1] = movmatrix_trans(Op::pack(p2, p3));
        }

#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
            const int r = (mt >> 2) * 16 + v_tok;
            const int c = ((mt & 3) << 1) + v_chunk;
            uint32_t a[4];
            ldmatrix_x4_trans(a, vt + r * 128 + ((c ^ (r & 7)) << 4));
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) Op::run(o[mt][nt], a, pb[nt][0], pb[nt][1]);
        }

        // Refill this stage with the page STAGES ahead.
        if (i + STAGES < n_my) {
            if (valid < 16) fence_proxy_async_smem();  // generic writes above, TMA write next
            __syncwarp();
            const long long id = __shfl_sync(0xffffffffu, my_id, i + STAGES);
            if (lane == 0) {
                fence_proxy_async_smem();
                const uint32_t bar = bar0 + 8 * st;
                mbar_arrive_expect_tx(bar, Shape::kStageBytes);
                tma_load_5d(kt, &kmap, 0, 0, 0, h, static_cast<int>(id), bar);
                tma_load_5d(vt, &vmap, 0, 0, 0, h, static_cast<int>(id), bar);
            }
        }
    }

    if (failed) {
        // Drain loads still in flight (bounded) before the stage memory is reused.
        const int last = i + STAGES < n_my ? i + STAGES : n_my;
        for (int j = i; j < last; ++j) mbar_wait_bounded(bar0 + 8 * (j % STAGES), (j / STAGES) & 1);
        if (lane == 0) {
            atomicOr(&g_device_status, kStatusWaitTimeout);
            atomicOr(&cta_bad, 2);
        }
    }

#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int off = 4; off < 32; off <<= 1)
                l_run[nt][j] += __shfl_xor_sync(0xffffffffu, l_run[nt][j], off);
        }
    }

    __syncthreads();  // every warp is done with its stages: reuse them for the merge
    float* red = reinterpret_cast<float*>(wsm);
    float* red_m = red + Shape::kQRows * Shape::kRedStride;
    float* red_l = red_m + Shape::kQRows;
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int d = mt * 16 + (lane >> 2);
            const int q = nt * 8 + 2 * (lane & 3);
            red[q * Shape::kRedStride + d] = o[mt][nt][0];
            red[(q + 1) * Shape::kRedStride + d] = o[mt][nt][1];
            red[q * Shape::kRedStride + d + 8] = o[mt][nt][2];
            red[(q + 1) * Shape::kRedStride + d + 8] = o[mt][nt][3];
        }
    }
    if (lane < 4) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int q = nt * 8 + 2 * lane;
            red_m[q] = m_run[nt][0];
            red_m[q + 1] = m_run[nt][1];
            red_l[q] = l_run[nt][0];
            red_l[q + 1] = l_run[nt][1];
        }
    }
    __syncthreads();
    if (cta_bad) {
        if (single) write_group_constant<T>(p, b, h, __int_as_float(0x7fffffff));
        else write_group_partial_nan(p, b, h, split);
        return;
    }

    T* out = static_cast<T*>(p.out);
    const int total = p.group * D;
    for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
        const int g = idx / D;
        const int d = idx - g * D;
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < NWARPS; ++w) {
            const float* wm = reinterpret_cast<const float*>(smem + w * Shape::kWarpBytes) +
                              Shape::kQRows * Shape::kRedStride;
            mx = fmaxf(mx, wm[g]);
        }
        float den = 0.0f;
        float num = 0.0f;
#pragma unroll
        for (int w = 0; w < NWARPS; ++w) {
            const float* wr = reinterpret_cast<const float*>(smem + w * Shape::kWarpBytes);
            const float* wm = wr + Shape::kQRows * Shape::kRedStride;
            const float f = fast_exp2(wm[g] - mx);
            den += f * wm[Shape::kQRows + g];
            num += f * wr[g * Shape::kRedStride + d];
        }
        const float value = num / den;
        if (single) {
            out[b * p.out_stride_seq + static_cast<int64_t>(h * p.group + g) * p.out_stride_head + d] =
                from_float<T>(value);
        } else {
            const int64_t row = (static_cast<int64_t>(b) * p.q_heads + h * p.group + g) * p.max_splits + split;
            p.part_o[row * D + d] = value;
            if (d == 0) p.part_lse[row] = mx + log2f(den);
        }
    }
}

}  // namespace mv
