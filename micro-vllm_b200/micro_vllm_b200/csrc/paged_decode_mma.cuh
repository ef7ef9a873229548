// Paged GQA decode on sm_100a: TMA page staging + tensor-core (mma.sync) tiles.
//
// The unit of work is one 16-token page of one KV head h of one sequence b.
// All query heads of h's GQA group are processed together, so each K/V page
// crosses HBM once (the reference kernel re-reads it once per query head:
// online_attention.cuh:112-115).
//
// Per page, one warp computes (WarpPageAttention below):
//   S^T[16 tok, 8 q] = K_page[16 x D] . Q^T         mma m16n8k16, A = K via ldmatrix
//   online softmax on the fragment (exp2 domain, quad shuffles for the max)
//   P^T fragment from S's accumulator by movmatrix.trans (no shared memory)
//   O^T[D, 8 q] += V_page^T[D x 16 tok] . P^T       mma m16n8k16, A = V via ldmatrix.trans
// The GQA group (<= 8 per n-tile, two n-tiles for groups up to 16) is the mma
// N dimension, so a group of 7 wastes one column of eight; D is the M dimension
// of the P.V product.
//
// Pages reach shared memory through each warp's own STAGES-deep ring: one lane
// issues two 5-D tiled TMA loads per page (the K page and the V page of head h,
// each block_size x D, 128-byte swizzled) that complete on the stage's mbarrier.
//
// Two schedules share that per-page code:
//  * paged_decode_mma_kernel -- one CTA per (split, KV head, sequence); warps
//    interleave the split's pages and merge through shared memory; a separate
//    merge pass combines splits.
//  * paged_decode_persistent_kernel -- one resident grid; the pages of the whole
//    batch, laid out (sequence, KV head, page), are cut into equal contiguous
//    ranges, one per warp (stream-K style), so every warp streams the same
//    number of bytes whatever the length mix. A warp's range covers whole
//    (sequence, head) segments, written as final output, plus at most two cut
//    segments at its ends, written as partials for the merge pass.
#pragma once

#include <cooperative_groups.h>

#include "mv_device.cuh"
#include "paged_decode_merge.cuh"

namespace mv {

constexpr int kPageTokens = 16;  // block_size of the tensor-core kernels (the mma M)
// Pages each warp requests into L2 (bulk tensor prefetch, no shared memory)
// beyond its shared-memory ring. 0 disables it: measured on B200 with one
// resident page stream per warp, prefetching 8 pages ahead thrashed L2 and
// cost 20-45% of bandwidth.
#ifndef MV_PREFETCH_PAGES
#define MV_PREFETCH_PAGES 0
#endif
constexpr int kPrefetchPages = MV_PREFETCH_PAGES;

template <int D>
struct PageTile {
    static constexpr int kBytes = kPageTokens * D * 2;  // one K (or V) page of one head
    static_assert(D % 64 == 0, "pages are staged as 64-column (128-byte) swizzled boxes");
};

// One warp's online-softmax state over the pages of one (sequence, KV head).
template <typename T, int D, int NT>
struct WarpPageAttention {
    using Op = MmaOp<T>;
    static constexpr int KS = D / 16;

    uint32_t qf[KS][NT][2];  // Q as the mma B operand
    float m[NT][2];          // running max (exp2 domain) of queries nt*8 + 2*(lane%4) + {0,1}
    float l[NT][2];          // running denominators (this lane's tokens only until reduce_l)
    float o[KS][NT][4];      // O^T accumulator fragments

    __device__ __forceinline__ void reset() {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            m[nt][0] = m[nt][1] = -INFINITY;
            l[nt][0] = l[nt][1] = 0.0f;
#pragma unroll
            for (int mt = 0; mt < KS; ++mt) o[mt][nt][0] = o[mt][nt][1] = o[mt][nt][2] = o[mt][nt][3] = 0.0f;
        }
    }

    // Lane holds q[g][16 ks + 2(lane%4) + {0,1,8,9}] for g = nt*8 + lane/4 (0 beyond the group).
    __device__ __forceinline__ void load_q(const DecodeParams& p, int b, int h, int lane) {
        load_q_frags(p, b, h, lane, qf);
    }

    // The same into any fragment array (the loads are only issued: nothing
    // waits for them until the fragments are read).
    __device__ __forceinline__ static void load_q_frags(const DecodeParams& p, int b, int h, int lane,
                                                        uint32_t (&qf)[KS][NT][2]) {
        const uint16_t* qbase = static_cast<const uint16_t*>(p.q) + row_q_offset(p, b);
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

    // Rotate-half RoPE of the loaded query fragments at table row `pos`. Element
    // d pairs with d + D/2, which this lane holds in the same slot of k-step
    // ks + KS/2, so the rotation needs no data from other lanes.
    __device__ __forceinline__ void rope_q(const DecodeParams& p, int64_t pos, int lane) {
        const T* cos_row = static_cast<const T*>(p.rope_cos) + pos * D;
        const T* sin_row = static_cast<const T*>(p.rope_sin) + pos * D;
#pragma unroll
        for (int ks = 0; ks < KS / 2; ++ks) {
#pragma unroll
            for (int w = 0; w < 2; ++w) {
                const int d = ks * 16 + 2 * (lane & 3) + 8 * w;
                float c0[2], s0[2], c1[2], s1[2];
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    c0[e] = to_float<T>(cos_row[d + e]);
                    s0[e] = to_float<T>(sin_row[d + e]);
                    c1[e] = to_float<T>(cos_row[d + e + D / 2]);
                    s1[e] = to_float<T>(sin_row[d + e + D / 2]);
                }
#pragma unroll
                for (int nt = 0; nt < NT; ++nt) {
                    uint32_t lo = qf[ks][nt][w], hi = qf[ks + KS / 2][nt][w];
                    const T* lv = reinterpret_cast<const T*>(&lo);
                    const T* hv = reinterpret_cast<const T*>(&hi);
                    uint32_t nlo, nhi;
                    T* nl = reinterpret_cast<T*>(&nlo);
                    T* nh = reinterpret_cast<T*>(&nhi);
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const float x0 = to_float<T>(lv[e]), x1 = to_float<T>(hv[e]);
                        nl[e] = from_float<T>(rope_element<T>(x0, x1, c0[e], s0[e], true));
                        nh[e] = from_float<T>(rope_element<T>(x1, x0, c1[e], s1[e], false));
                    }
                    qf[ks][nt][w] = nlo;
                    qf[ks + KS / 2][nt][w] = nhi;
                }
            }
        }
    }

    // The staged page as mma A fragments: K for S^T = K Q^T, V^T (via .trans)
    // for O^T += V^T P^T. Loading them first frees the stage for the next TMA
    // load before any of the page's arithmetic runs.
    struct PageFrags {
        uint32_t k[KS][4];
        uint32_t v[KS][4];
    };

    // K tile at shared address kt, V tile at vt (vgen: its generic pointer);
    // `valid` tokens of 16 in use.
    __device__ __forceinline__ static void load_page(PageFrags& f, uint32_t kt, uint32_t vt, uint8_t* vgen,
                                                     int valid, int lane) {
        if (valid < kPageTokens) {
            // Slots past the context may hold anything (NaN included); P is 0 there,
            // but 0 * NaN is NaN, so clear those V rows before P.V.
            const int rows = kPageTokens - valid;
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
        const int k_slot = (lane & 7) + ((lane >> 3) & 1) * 8;  // A = K: matrices (rows, cols) 00,10,01,11
        const int k_chunk = lane >> 4;
        const int v_tok = (lane & 7) + ((lane >> 4) & 1) * 8;   // A = V^T via .trans
        const int v_chunk = (lane >> 3) & 1;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int r = (ks >> 2) * 16 + k_slot;
            const int c = ((ks & 3) << 1) + k_chunk;
            ldmatrix_x4(f.k[ks], kt + r * 128 + ((c ^ (r & 7)) << 4));
        }
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
            const int r = (mt >> 2) * 16 + v_tok;
            const int c = ((mt & 3) << 1) + v_chunk;
            ldmatrix_x4_trans(f.v[mt], vt + r * 128 + ((c ^ (r & 7)) << 4));
        }
    }

    // Online-softmax update with one page held in registers.
    __device__ __forceinline__ void attend(const PageFrags& f, int valid, float scale_log2, int lane) {
        float sc[NT][2][4];
        scores(f.k, sc);
        update(sc, f.v, valid, scale_log2, lane);
    }

    // The page's K tile as A fragments (lane layout of load_page).
    __device__ __forceinline__ static void load_k(uint32_t (&k)[KS][4], uint32_t kt, int lane) {
        const int k_slot = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int k_chunk = lane >> 4;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int r = (ks >> 2) * 16 + k_slot;
            const int c = ((ks & 3) << 1) + k_chunk;
            ldmatrix_x4(k[ks], kt + r * 128 + ((c ^ (r & 7)) << 4));
        }
    }

    // The page's V tile as transposed A fragments; slots past `valid` cleared first.
    __device__ __forceinline__ static void load_v(uint32_t (&v)[KS][4], uint32_t vt, uint8_t* vgen, int valid,
                                                  int lane) {
        if (valid < kPageTokens) {
            const int rows = kPageTokens - valid;
            for (int idx = lane; idx < (D / 64) * rows * 8; idx += 32) {
                const int chunk = idx & 7;
                const int rr = idx >> 3;
                const int half = rr / rows;
                const int slot = valid + (rr - half * rows);
                *reinterpret_cast<uint4*>(vgen + (half * 16 + slot) * 128 + chunk * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
            __syncwarp();
        }
        const int v_tok = (lane & 7) + ((lane >> 4) & 1) * 8;
        const int v_chunk = (lane >> 3) & 1;
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
            const int r = (mt >> 2) * 16 + v_tok;
            const int c = ((mt & 3) << 1) + v_chunk;
            ldmatrix_x4_trans(v[mt], vt + r * 128 + ((c ^ (r & 7)) << 4));
        }
    }

    // S^T = K Q^T for one page (two accumulator chains: even and odd k-steps
    // halve the dependent mma chain).
    __device__ __forceinline__ void scores(const uint32_t (&k)[KS][4], float (&sc)[NT][2][4]) const {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int c = 0; c < 2; ++c) sc[nt][c][0] = sc[nt][c][1] = sc[nt][c][2] = sc[nt][c][3] = 0.0f;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) Op::run(sc[nt][ks & 1], k[ks], qf[ks][nt][0], qf[ks][nt][1]);
        }
    }

    // Online-softmax update from one page's scores and its V fragments.
    __device__ __forceinline__ void update(const float (&sc)[NT][2][4], const uint32_t (&v)[KS][4], int valid,
                                           float scale_log2, int lane) {
        const int row0 = lane >> 2;  // token of accumulator rows c0/c1 (+8 for c2/c3)
        const bool v0 = row0 < valid;
        const bool v1 = row0 + 8 < valid;
        uint32_t pb[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const float x0 = v0 ? (sc[nt][0][0] + sc[nt][1][0]) * scale_log2 : -INFINITY;
            const float x1 = v0 ? (sc[nt][0][1] + sc[nt][1][1]) * scale_log2 : -INFINITY;
            const float x2 = v1 ? (sc[nt][0][2] + sc[nt][1][2]) * scale_log2 : -INFINITY;
            const float x3 = v1 ? (sc[nt][0][3] + sc[nt][1][3]) * scale_log2 : -INFINITY;
            float mx0 = fmaxf(x0, x2);
            float mx1 = fmaxf(x1, x3);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float mn0 = fmaxf(m[nt][0], mx0);
            const float mn1 = fmaxf(m[nt][1], mx1);
            const float a0 = fast_exp2(m[nt][0] - mn0);
            const float a1 = fast_exp2(m[nt][1] - mn1);
            m[nt][0] = mn0;
            m[nt][1] = mn1;
            const float p0 = fast_exp2(x0 - mn0);
            const float p1 = fast_exp2(x1 - mn1);
            const float p2 = fast_exp2(x2 - mn0);
            const float p3 = fast_exp2(x3 - mn1);
            l[nt][0] = l[nt][0] * a0 + (p0 + p2);
            l[nt][1] = l[nt][1] * a1 + (p1 + p3);
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
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) Op::run(o[mt][nt], v[mt], pb[nt][0], pb[nt][1]);
        }
    }

    // Sum the denominators over the eight lanes that share a query pair.
    __device__ __forceinline__ void reduce_l() {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
#pragma unroll
                for (int off = 4; off < 32; off <<= 1) l[nt][j] += __shfl_xor_sync(0xffffffffu, l[nt][j], off);
            }
        }
    }

    // out[b, h*G + q, :] = O / l for q < group (after reduce_l).
    __device__ __forceinline__ void store_final(const DecodeParams& p, int b, int h, int lane) const {
        T* out = static_cast<T*>(p.out) + b * p.out_stride_seq;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int q = nt * 8 + 2 * (lane & 3) + j;
                if (q >= p.group) continue;
                const float inv = 1.0f / l[nt][j];
                T* row = out + static_cast<int64_t>(h * p.group + q) * p.out_stride_head;
#pragma unroll
                for (int mt = 0; mt < KS; ++mt) {
                    const int d = mt * 16 + (lane >> 2);
                    row[d] = from_float<T>(o[mt][nt][j] * inv);
                    row[d + 8] = from_float<T>(o[mt][nt][j + 2] * inv);
                }
            }
        }
    }

    // Normalised partial [8*NT][D] and its log2-sum-exp [8*NT] (after reduce_l).
    __device__ __forceinline__ void store_partial(float* po, float* plse, int group, int lane) const {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int q = nt * 8 + 2 * (lane & 3) + j;
                if (q >= group) continue;
                const float inv = 1.0f / l[nt][j];
                float* row = po + q * D;
#pragma unroll
                for (int mt = 0; mt < KS; ++mt) {
                    const int d = mt * 16 + (lane >> 2);
                    row[d] = o[mt][nt][j] * inv;
                    row[d + 8] = o[mt][nt][j + 2] * inv;
                }
                if ((lane >> 2) == 0) plse[q] = m[nt][j] + log2f(l[nt][j]);
            }
        }
    }

    // The same into rows `row_stride` floats apart (log2-sum-exps `lse_stride`
    // apart): query row q of one split of the split-KV partial layout.
    __device__ __forceinline__ void store_partial_strided(float* po, float* plse, int64_t row_stride,
                                                          int64_t lse_stride, int group, int lane) const {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                const int q = nt * 8 + 2 * (lane & 3) + j;
                if (q >= group) continue;
                const float inv = 1.0f / l[nt][j];
                float* row = po + q * row_stride;
#pragma unroll
                for (int mt = 0; mt < KS; ++mt) {
                    const int d = mt * 16 + (lane >> 2);
                    row[d] = o[mt][nt][j] * inv;
                    row[d + 8] = o[mt][nt][j + 2] * inv;
                }
                if ((lane >> 2) == 0) plse[q * lse_stride] = m[nt][j] + log2f(l[nt][j]);
            }
        }
    }

    __device__ __forceinline__ void store_partial_nan(float* po, float* plse, int group, int lane) const {
        const float nan = __int_as_float(0x7fffffff);
        for (int idx = lane; idx < group * D; idx += 32) po[idx] = nan;
        if (lane < group) plse[lane] = nan;
    }
};

// CUDA-core variant of the per-page math (MV_FLAG_CUDA_CORE_MATH, GQA group
// <= 8, head_dim 64/128), kept to compare with the tensor-core tile on the
// same TMA pipeline and grid: fp32 FMA dot products straight from the staged
// page in shared memory, q in shared memory as fp32.
//   S: lane = (token t = lane % 16, half of the row lane / 16); the halves'
//      sums meet through one shuffle; the online softmax runs per token lane.
//   P.V: lane = D / 32 columns of O for all eight query heads; P of the page
//      goes through a 16 x 8 fp32 buffer of the warp in shared memory.
// P stays fp32 (the tensor-core tile rounds it to the element type).
template <typename T, int D>
struct WarpPageFma {
    static constexpr int kG = 8;                  // query heads per tile (q rows past the group are 0)
    static constexpr int kHalfChunks = D / 16;    // 16-byte chunks in half a row
    static constexpr int kCols = D / 32;          // O columns per lane
    static constexpr int kQBytes = kG * D * 4;    // q of the group, fp32
    static constexpr int kPBytes = 16 * kG * 4;   // P of one page, per warp

    float m[kG];          // running max (exp2 domain), the same on every lane
    float l[kG];          // denominators: lanes 0..15 hold their token's share
    float o[kG][kCols];   // O[g][lane * kCols + j]

    __device__ __forceinline__ void reset() {
#pragma unroll
        for (int g = 0; g < kG; ++g) {
            m[g] = -INFINITY;
            l[g] = 0.0f;
#pragma unroll
            for (int j = 0; j < kCols; ++j) o[g][j] = 0.0f;
        }
    }

    // q rows h*G + g of row b into qs[g][d] as fp32 (0 for g >= group), rotated
    // at table row `pos` when rope is set; every thread of the CTA takes part
    // (the caller synchronises the CTA afterwards).
    __device__ static void load_q(const DecodeParams& p, int b, int h, int64_t pos, bool rope, float* qs) {
        const T* qbase = static_cast<const T*>(p.q) + row_q_offset(p, b);
        for (int idx = threadIdx.x; idx < kG * D; idx += blockDim.x) {
            const int g = idx / D;
            const int d = idx - g * D;
            float v = 0.0f;
            if (g < p.group) {
                const T* row = qbase + static_cast<int64_t>(h * p.group + g) * p.q_stride_head;
                v = to_float<T>(row[d]);
                if (rope) {
                    const bool first = d < D / 2;
                    const float partner = to_float<T>(row[first ? d + D / 2 : d - D / 2]);
                    const float c = to_float<T>(static_cast<const T*>(p.rope_cos)[pos * D + d]);
                    const float sn = to_float<T>(static_cast<const T*>(p.rope_sin)[pos * D + d]);
                    v = rope_element<T>(v, partner, c, sn, first);
                }
            }
            qs[idx] = v;
        }
    }

    static __device__ __forceinline__ void unpack8(const uint4& raw, float (&f)[8]) {
        const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
        for (int i = 0; i < 8; ++i) f[i] = to_float<T>(e[i]);
    }

    // One page: K tile at kt, V tile at vt (generic pointers into the stage,
    // 128-byte swizzled 16 x 64 boxes), `valid` of its 16 tokens in use.
    __device__ __forceinline__ void attend(const uint8_t* kt, const uint8_t* vt, const float* qs, float* pbuf,
                                           int valid, float scale_log2, int lane) {
        const int t = lane & 15;
        const int half = lane >> 4;
        float s[kG];
#pragma unroll
        for (int g = 0; g < kG; ++g) s[g] = 0.0f;
#pragma unroll
        for (int j = 0; j < kHalfChunks; ++j) {
            const int gc = half * kHalfChunks + j;   // row chunk: dims 8 gc .. 8 gc + 7
            const int c = gc & 7;
            float kf[8];
            unpack8(*reinterpret_cast<const uint4*>(kt + (gc >> 3) * 2048 + t * 128 + ((c ^ (t & 7)) << 4)), kf);
#pragma unroll
            for (int g = 0; g < kG; ++g) {
                const float4 q0 = *reinterpret_cast<const float4*>(qs + g * D + gc * 8);
                const float4 q1 = *reinterpret_cast<const float4*>(qs + g * D + gc * 8 + 4);
                float acc = s[g];
                acc = fmaf(kf[0], q0.x, acc);
                acc = fmaf(kf[1], q0.y, acc);
                acc = fmaf(kf[2], q0.z, acc);
                acc = fmaf(kf[3], q0.w, acc);
                acc = fmaf(kf[4], q1.x, acc);
                acc = fmaf(kf[5], q1.y, acc);
                acc = fmaf(kf[6], q1.z, acc);
                acc = fmaf(kf[7], q1.w, acc);
                s[g] = acc;
            }
        }
        const bool in = t < valid;
        float a[kG];
        float pv[kG];
#pragma unroll
        for (int g = 0; g < kG; ++g) {
            const float sum = s[g] + __shfl_xor_sync(0xffffffffu, s[g], 16);   // every lane takes part
            const float x = in ? sum * scale_log2 : -INFINITY;
            float mx = x;
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[g], mx);   // finite: token 0 of a page is always in use
            a[g] = fast_exp2(m[g] - mn);
            pv[g] = in ? fast_exp2(x - mn) : 0.0f;
            m[g] = mn;
            l[g] = l[g] * a[g] + (half == 0 ? pv[g] : 0.0f);
        }
        if (half == 0) {
            *reinterpret_cast<float4*>(pbuf + t * kG) = make_float4(pv[0], pv[1], pv[2], pv[3]);
            *reinterpret_cast<float4*>(pbuf + t * kG + 4) = make_float4(pv[4], pv[5], pv[6], pv[7]);
        }
        __syncwarp();
#pragma unroll
        for (int g = 0; g < kG; ++g)
#pragma unroll
            for (int j = 0; j < kCols; ++j) o[g][j] *= a[g];
        const int d0 = lane * kCols;
        const int c = (d0 & 63) >> 3;
        const uint8_t* vcol = vt + (d0 >> 6) * 2048 + (d0 & 7) * 2;
        for (int tt = 0; tt < valid; ++tt) {
            const float4 p0 = *reinterpret_cast<const float4*>(pbuf + tt * kG);
            const float4 p1 = *reinterpret_cast<const float4*>(pbuf + tt * kG + 4);
            const uint8_t* src = vcol + tt * 128 + ((c ^ (tt & 7)) << 4);
            float vf[kCols];
            if constexpr (kCols == 4) {
                const uint2 raw = *reinterpret_cast<const uint2*>(src);
                const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
                for (int j = 0; j < 4; ++j) vf[j] = to_float<T>(e[j]);
            } else {
                const uint32_t raw = *reinterpret_cast<const uint32_t*>(src);
                const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
                for (int j = 0; j < kCols; ++j) vf[j] = to_float<T>(e[j]);
            }
            const float pw[kG] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
            for (int g = 0; g < kG; ++g)
#pragma unroll
                for (int j = 0; j < kCols; ++j) o[g][j] = fmaf(pw[g], vf[j], o[g][j]);
        }
        __syncwarp();   // every lane read pbuf before the next page writes it
    }

    // Full denominators on every lane (lanes 16..31 contribute 0).
    __device__ __forceinline__ void reduce_l() {
#pragma unroll
        for (int g = 0; g < kG; ++g)
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) l[g] += __shfl_xor_sync(0xffffffffu, l[g], off);
    }

    // The warp's state into the CTA merge buffers (the tensor-core tile's format).
    __device__ __forceinline__ void store_red(float* red, float* red_m, float* red_l, int stride, int lane) const {
#pragma unroll
        for (int g = 0; g < kG; ++g)
#pragma unroll
            for (int j = 0; j < kCols; ++j) red[g * stride + lane * kCols + j] = o[g][j];
        if (lane == 0) {
#pragma unroll
            for (int g = 0; g < kG; ++g) {
                red_m[g] = m[g];
                red_l[g] = l[g];
            }
        }
    }
};

// ------------------------------------------------------- split-grid kernel

// After a CTA wrote its split's partial: count it in, and if it is the
// segment's last split, merge the segment. The counter wraps back to 0 at the
// last arrival (atomicInc), so it is zero again for the next call.
template <typename T>
__device__ void arrive_and_merge(const DecodeParams& p, int b, int h, int splits, float* weights,
                                 int* flag) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned old = atomicInc(p.counters + b * p.kv_heads + h, static_cast<unsigned>(splits - 1));
        *flag = old == static_cast<unsigned>(splits - 1);
    }
    __syncthreads();
    if (*flag) {
        __threadfence();
        if ((p.head_dim == 64 || p.head_dim == 128) && splits <= kSegmentWarpBatch &&
            p.group <= 2 * static_cast<int>(blockDim.x >> 5))
            merge_segment_warps<T>(p, b, h, splits);
        else
            merge_segment<T>(p, b, h, splits, weights);
    }
}

template <int D, int NT, int NWARPS, int STAGES>
struct MmaDecodeShape {
    static constexpr int kTileBytes = PageTile<D>::kBytes;
    static constexpr int kStageBytes = 2 * kTileBytes;
    static constexpr int kWarpBytes = STAGES * kStageBytes;
    static constexpr int kSmemBytes = NWARPS * kWarpBytes + 1024;  // + 1 KiB for alignment
    static constexpr int kQRows = 8 * NT;
    static constexpr int kRedStride = D + 4;
    static constexpr int kRedBytes = (kQRows * kRedStride + 2 * kQRows) * 4;
    static constexpr int kMaxPagesPerSplit = 32 * NWARPS;  // one page ID per lane per warp
    static_assert(kRedBytes <= kWarpBytes, "warp merge buffer must fit the warp's stages");
};

// Before the grid-dependency wait, a CTA of the first wave can bring its first
// pages into L2, so its first TMA loads after the wait hit L2 instead of
// waiting on DRAM while the previous kernel (a merge pass, the previous
// layer's step) finishes. The length and the page IDs may still be written by
// that kernel, so they are read through L2 (load_index_l2_hint) and used only
// as prefetch addresses: an L2 prefetch changes no data, an ID outside the pool
// is skipped, and every value the kernel computes with is read again after the
// wait.
template <int NWARPS>
__device__ __forceinline__ void prewait_page_prefetch(const DecodeParams& p, const CUtensorMap* kmap,
                                                      const CUtensorMap* vmap, int split, int h, int b, int warp,
                                                      int lane) {
    if (!p.context_lens || p.contiguous || p.q_tokens != 1) return;
    const int64_t len = load_index_l2_hint(p.context_lens, p.lens_i64, b);
    if (len <= 0 || len > p.max_context_len || len > p.blocks_per_seq * p.block_size) return;
    const int64_t pages = (len + kPageTokens - 1) / kPageTokens;
    const int64_t begin = split_begin(p, split);
    if (begin >= pages) return;
    const int64_t raw_end = begin + split_pages(p, split);
    const int n = static_cast<int>((raw_end < pages ? raw_end : pages) - begin);
    const int n_my = warp < n ? (n - warp + NWARPS - 1) / NWARPS : 0;
    if (lane < n_my && lane < p.prewait_pages) {
        const int64_t id = load_index_l2_hint(p.block_table, p.table_i64,
                                              b * p.table_stride + begin + warp + lane * NWARPS);
        if (id >= 0 && id < p.num_blocks) {
            tma_prefetch_l2_5d(kmap, 0, 0, 0, h, static_cast<int>(id));
            tma_prefetch_l2_5d(vmap, 0, 0, 0, h, static_cast<int>(id));
        }
    }
}

// Shared memory the CUDA-core variant adds after the stages: q of the group
// (fp32) and each warp's P buffer.
template <typename T, int D, int NWARPS>
constexpr int fma_extra_smem() {
    return WarpPageFma<T, D>::kQBytes + NWARPS * WarpPageFma<T, D>::kPBytes;
}

template <typename T, int D, int NT, int NWARPS, int STAGES, bool FMA = false>
__global__ void __launch_bounds__(NWARPS * 32)
paged_decode_mma_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap) {
    using Shape = MmaDecodeShape<D, NT, NWARPS, STAGES>;
    using Warp = WarpPageAttention<T, D, NT>;
    static_assert(!FMA || (NT == 1 && (D == 64 || D == 128)), "CUDA-core variant: group <= 8, head_dim 64/128");

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[NWARPS][STAGES];
    __shared__ int warp_flags[NWARPS];  // 1: corrupted page ID, 2: a wait gave up
    __shared__ int cta_last;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    int split, h, b;
    if (p.first_pages > 0) {
        // Split-major order over the (splits, kv_heads, batch) grid: linear
        // block index = (split * kv_heads + h) * batch + b.
        const int64_t lin = blockIdx.x + static_cast<int64_t>(gridDim.x) *
                                             (blockIdx.y + static_cast<int64_t>(gridDim.y) * blockIdx.z);
        b = static_cast<int>(lin % gridDim.z);
        h = static_cast<int>((lin / gridDim.z) % gridDim.y);
        split = static_cast<int>(lin / (static_cast<int64_t>(gridDim.z) * gridDim.y));
    } else {
        split = blockIdx.x;
        h = blockIdx.y;
        b = blockIdx.z;
    }

    if (p.prewait_ctas > 0 &&
        blockIdx.x + static_cast<int64_t>(gridDim.x) * (blockIdx.y + static_cast<int64_t>(gridDim.y) * blockIdx.z) <
            p.prewait_ctas)
        prewait_page_prefetch<NWARPS>(p, &kmap, &vmap, split, h, b, warp, lane);
    wait_for_prior_grid();
    allow_next_grid();
    const SeqSplit seq = seq_split(p, b);
    if (split >= seq.splits) return;
    if (seq.state != 0) {
        if (p.new_key) append_row_direct<T>(p, b, h, seq.len);
        write_group_constant<T>(p, b, h, seq.state == 1 ? 0.0f : __int_as_float(0x7fffffff));
        return;
    }
    // Fused RoPE needs a table row for the step's position. Without one the
    // group takes the corrupted-page path below (no loads, NaN result through
    // the split partials) and nothing is appended.
    const bool rope_missing = p.rope_cos && seq.len - 1 >= p.rope_rows;
    const bool single = seq.splits == 1;

    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    int64_t page_begin, page_end;
    split_range(p, seq, split, &page_begin, &page_end);
    const int cta_pages = static_cast<int>(page_end - page_begin);
    const int n_my = (warp < cta_pages && !rope_missing) ? (cta_pages - warp + NWARPS - 1) / NWARPS : 0;

    // Page IDs of this warp's pages: lane i holds page warp + i * NWARPS of the run.
    // A corrupted ID (outside the pool) is never loaded; the group becomes NaN.
    long long my_id = 0;
    bool bad = false;
    if (lane < n_my) {
        const int64_t page = page_begin + warp + lane * NWARPS;
        // A contiguous cache's "page" is a run of 16 tokens: its index is its ID.
        my_id = p.contiguous ? page
                             : load_index(p.block_table, p.table_i64, row_seq(p, b) * p.table_stride + page);
        bad = !p.contiguous && (my_id < 0 || my_id >= p.num_blocks);
    }
    const bool any_bad_id = __any_sync(0xffffffffu, bad);
    if (any_bad_id && lane == 0) report_bad_page_id();
    const bool warp_has_bad = any_bad_id || rope_missing;
    const uint32_t bar0 = smem_addr(&bars[warp][0]);
    if (lane == 0) {
#pragma unroll
        for (int st = 0; st < STAGES; ++st) mbar_init(bar0 + 8 * st, 1);
    }
    fence_mbar_init();
    __syncwarp();

    uint8_t* wsm = smem + warp * Shape::kWarpBytes;
    const uint32_t wsm_addr = smem_addr(wsm);

    // Fill page i of this warp into its stage (every lane calls; lane 0 issues).
    auto issue = [&](int i) {
        const long long id = __shfl_sync(0xffffffffu, my_id, i);
        const bool ok = id >= 0 && id < p.num_blocks;
        if (lane == 0) {
            const int st = i % STAGES;
            const uint32_t bar = bar0 + 8 * st;
            if (ok) {
                const uint32_t dst = wsm_addr + st * Shape::kStageBytes;
                mbar_arrive_expect_tx(bar, Shape::kStageBytes);
                if (p.contiguous) {
                    // Map (d%64, token, d/64, head, sequence): tokens past the cache read as 0.
                    const int seq = static_cast<int>(row_seq(p, b));
                    tma_load_5d(dst, &kmap, 0, static_cast<int>(id) * kPageTokens, 0, h, seq, bar);
                    tma_load_5d(dst + Shape::kTileBytes, &vmap, 0, static_cast<int>(id) * kPageTokens, 0, h, seq, bar);
                } else {
                    tma_load_5d(dst, &kmap, 0, 0, 0, h, static_cast<int>(id), bar);
                    tma_load_5d(dst + Shape::kTileBytes, &vmap, 0, 0, 0, h, static_cast<int>(id), bar);
                }
            } else {
                // No load for a corrupted ID; complete the phase so the ring stays in step.
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
            }
        }
    };

    const int prologue = n_my < STAGES ? n_my : STAGES;
    for (int i = 0; i < prologue; ++i) issue(i);
    for (int i = prologue; kPrefetchPages > 0 && i < n_my && i < STAGES + kPrefetchPages; ++i) {
        const long long id = __shfl_sync(0xffffffffu, my_id, i);
        if (lane == 0 && id >= 0 && id < p.num_blocks) {
            tma_prefetch_l2_5d(&kmap, 0, 0, 0, h, static_cast<int>(id));
            tma_prefetch_l2_5d(&vmap, 0, 0, 0, h, static_cast<int>(id));
        }
    }

    // Fused append: the warp that attends the sequence's last page holds the
    // new K/V row (16-byte chunks; lanes 0..D/8-1 K, the next D/8 V, wrapping
    // for D = 256) and writes it into that page after the page's TMA load
    // landed -- into the staged tile, which this warp then reads, and into the
    // pool. Only this CTA reads the last page, so nothing else can see the old row.
    constexpr int kRowChunks = D / 8;
    constexpr int kNewPerLane = (2 * kRowChunks + 31) / 32;
    int append_at = -1;  // loop index of the last page in this warp, or -1
    uint4 new_rows[kNewPerLane];
    if (p.new_key && split == seq.splits - 1 && !rope_missing) {
        const int rel = static_cast<int>(seq.pages - 1 - page_begin);
        if (rel % NWARPS == warp) {
            append_at = rel / NWARPS;
#pragma unroll
            for (int j = 0; j < kNewPerLane; ++j) {
                const int c = lane + 32 * j;
                if (c < 2 * kRowChunks) {
                    const int which = c >= kRowChunks;
                    const int cc = c - which * kRowChunks;
                    const int64_t* st = which ? p.new_value_stride : p.new_key_stride;
                    const uint4* row = reinterpret_cast<const uint4*>(
                        static_cast<const uint16_t*>(which ? p.new_value : p.new_key) + b * st[0] + h * st[1]);
                    new_rows[j] = row[cc];
                    if (p.rope_cos && !which) {
                        // The K chunk pairs with the chunk D/2 away (rotate-half).
                        const int64_t t = (seq.len - 1) * kRowChunks + cc;
                        new_rows[j] = rope_chunk<T>(new_rows[j], row[cc ^ (kRowChunks / 2)],
                                                    reinterpret_cast<const uint4*>(p.rope_cos)[t],
                                                    reinterpret_cast<const uint4*>(p.rope_sin)[t],
                                                    cc < kRowChunks / 2);
                    }
                }
            }
        }
    }

    std::conditional_t<FMA, WarpPageFma<T, D>, Warp> w;
    float* fma_q = reinterpret_cast<float*>(smem + NWARPS * Shape::kWarpBytes);
    float* fma_p = fma_q + 8 * D + warp * 16 * 8;
    if constexpr (FMA) {
        WarpPageFma<T, D>::load_q(p, b, h, seq.len - 1, p.rope_cos && !rope_missing, fma_q);
        __syncthreads();
    } else {
        w.load_q(p, b, h, lane);
        if (p.rope_cos && !rope_missing) w.rope_q(p, seq.len - 1, lane);
    }
    w.reset();

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
        const int64_t left = seq.len - page * kPageTokens;
        const int valid = left < kPageTokens ? static_cast<int>(left) : kPageTokens;
        const bool page_ok = !warp_has_bad || __shfl_sync(0xffffffffu, !bad, i);
        if (i == append_at && page_ok) {
            const long long id = __shfl_sync(0xffffffffu, my_id, i);
            const int slot = valid - 1;
            uint8_t* tiles = wsm + st * Shape::kStageBytes;
#pragma unroll
            for (int j = 0; j < kNewPerLane; ++j) {
                const int c = lane + 32 * j;
                if (c < 2 * kRowChunks) {
                    const int which = c >= kRowChunks;
                    const int cc = c - which * kRowChunks;
                    const int r = (cc >> 3) * 16 + slot;  // 64-column box, then token
                    *reinterpret_cast<uint4*>(tiles + which * Shape::kTileBytes + r * 128 +
                                              (((cc & 7) ^ (r & 7)) << 4)) = new_rows[j];
                    uint16_t* pool = const_cast<uint16_t*>(
                        static_cast<const uint16_t*>(which ? p.v_cache : p.k_cache));
                    reinterpret_cast<uint4*>(pool + ((id * p.kv_heads + h) * kPageTokens + slot) * D)[cc] =
                        new_rows[j];
                }
            }
            __syncwarp();
        }
        if constexpr (FMA) {
            // The math reads the stage itself: refill it afterwards.
            if (page_ok)
                w.attend(wsm + st * Shape::kStageBytes, wsm + st * Shape::kStageBytes + Shape::kTileBytes, fma_q,
                         fma_p, valid, p.scale_log2, lane);
            if (i + STAGES < n_my) {
                fence_proxy_async_smem();
                __syncwarp();
                issue(i + STAGES);
            }
        } else {
        typename Warp::PageFrags frags;
        if (page_ok) Warp::load_page(frags, kt, vt, wsm + st * Shape::kStageBytes + Shape::kTileBytes, valid, lane);

        // The page is in registers: refill its stage before the arithmetic.
        if (i + STAGES < n_my) {
            fence_proxy_async_smem();  // this lane's shared reads/writes before the TMA write
            __syncwarp();
            issue(i + STAGES);
            const int ahead = i + STAGES + kPrefetchPages;
            const long long pf = __shfl_sync(0xffffffffu, my_id, ahead & 31);
            if (kPrefetchPages > 0 && lane == 0 && ahead < n_my && pf >= 0 && pf < p.num_blocks) {
                tma_prefetch_l2_5d(&kmap, 0, 0, 0, h, static_cast<int>(pf));
                tma_prefetch_l2_5d(&vmap, 0, 0, 0, h, static_cast<int>(pf));
            }
        }
        if (page_ok) w.attend(frags, valid, p.scale_log2, lane);
        }
    }

    if (failed) {
        // Drain loads still in flight (bounded) before the stage memory is reused.
        const int last = i + STAGES < n_my ? i + STAGES : n_my;
        for (int j = i; j < last; ++j) mbar_wait_bounded(bar0 + 8 * (j % STAGES), (j / STAGES) & 1);
        if (lane == 0) atomicOr(&g_device_status, kStatusWaitTimeout);
    }
    if (lane == 0) warp_flags[warp] = (failed ? 2 : 0) | (warp_has_bad ? 1 : 0);
    w.reduce_l();

    __syncthreads();  // every warp is done with its stages: reuse them for the merge
    float* red = reinterpret_cast<float*>(wsm);
    float* red_m = red + Shape::kQRows * Shape::kRedStride;
    float* red_l = red_m + Shape::kQRows;
    if constexpr (FMA) {
        w.store_red(red, red_m, red_l, Shape::kRedStride, lane);
    } else {
#pragma unroll
    for (int mt = 0; mt < Warp::KS; ++mt) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int d = mt * 16 + (lane >> 2);
            const int q = nt * 8 + 2 * (lane & 3);
            red[q * Shape::kRedStride + d] = w.o[mt][nt][0];
            red[(q + 1) * Shape::kRedStride + d] = w.o[mt][nt][1];
            red[q * Shape::kRedStride + d + 8] = w.o[mt][nt][2];
            red[(q + 1) * Shape::kRedStride + d + 8] = w.o[mt][nt][3];
        }
    }
    if (lane < 4) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int q = nt * 8 + 2 * lane;
            red_m[q] = w.m[nt][0];
            red_m[q + 1] = w.m[nt][1];
            red_l[q] = w.l[nt][0];
            red_l[q + 1] = w.l[nt][1];
        }
    }
    }
    __syncthreads();
    int cta_bad = 0;
#pragma unroll
    for (int v = 0; v < NWARPS; ++v) cta_bad |= warp_flags[v];
    if (cta_bad) {
        if (single) {
            write_group_constant<T>(p, b, h, __int_as_float(0x7fffffff));
        } else {
            write_group_partial_nan(p, b, h, split);
            if (p.fused_merge) arrive_and_merge<T>(p, b, h, seq.splits, reinterpret_cast<float*>(smem), &cta_last);
        }
        return;
    }

    T* out = static_cast<T*>(p.out);
    const int total = p.group * D;
    for (int idx = threadIdx.x; idx < total; idx += blockDim.x) {
        const int g = idx / D;
        const int d = idx - g * D;
        float mx = -INFINITY;
#pragma unroll
        for (int v = 0; v < NWARPS; ++v) {
            const float* wm = reinterpret_cast<const float*>(smem + v * Shape::kWarpBytes) +
                              Shape::kQRows * Shape::kRedStride;
            mx = fmaxf(mx, wm[g]);
        }
        float den = 0.0f;
        float num = 0.0f;
#pragma unroll
        for (int v = 0; v < NWARPS; ++v) {
            const float* wr = reinterpret_cast<const float*>(smem + v * Shape::kWarpBytes);
            const float* wm = wr + Shape::kQRows * Shape::kRedStride;
            const float f = fast_exp2(wm[g] - mx);
            den += f * wm[Shape::kQRows + g];
            num += f * wr[g * Shape::kRedStride + d];
        }
        const float value = num / den;
        if (single) {
            out[row_out_offset(p, b) + static_cast<int64_t>(h * p.group + g) * p.out_stride_head + d] =
                from_float<T>(value);
        } else {
            const int64_t row = (static_cast<int64_t>(b) * p.q_heads + h * p.group + g) * p.max_splits + split;
            p.part_o[row * D + d] = value;
            if (d == 0) p.part_lse[row] = mx + log2f(den);
        }
    }
    if (!single && p.fused_merge) {
        __syncthreads();  // the warps' merge buffers are read: reuse shared memory for weights
        arrive_and_merge<T>(p, b, h, seq.splits, reinterpret_cast<float*>(smem), &cta_last);
    }
}

// --------------------------------------------------------- persistent kernel

template <int D, int NWARPS, int STAGES>
struct PersistentShape {
    static constexpr int kTileBytes = PageTile<D>::kBytes;
    static constexpr int kStageBytes = 2 * kTileBytes;
    static constexpr int kWarpBytes = STAGES * kStageBytes;
    static constexpr int kStageRegion = NWARPS * kWarpBytes;
    // + prefix array of (batch + 1) int64, + 1 KiB for alignment
    static __host__ __device__ constexpr int smem_bytes(int batch) {
        return kStageRegion + (batch + 1) * 8 + 1024;
    }
};

// Global page index -> (sequence, head, page). Segments are laid out
// sequence-major, then KV head: segment (b, h) holds pages
// [Hkv*prefix[b] + h*pages_b, + pages_b) of the batch's page space.
struct PageRef {
    int seg;      // b * kv_heads + h, or -1 past the warp's range
    int page;     // page index within the sequence
    int id;       // physical page, -1 if the table entry is outside the pool
    int meta;     // valid tokens (bits 0..7) | last page of its segment (bit 8)
};

__device__ __forceinline__ PageRef locate_page(const DecodeParams& p, const int64_t* prefix,
                                               int64_t g) {
    // Largest b with kv_heads * prefix[b] <= g.
    int lo = 0;
    int hi = p.batch;  // prefix[batch] * kv_heads > g always
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (p.kv_heads * prefix[mid] <= g) lo = mid;
        else hi = mid;
    }
    const int b = lo;
    const int64_t pages_b = prefix[b + 1] - prefix[b];
    const int64_t r = g - p.kv_heads * prefix[b];
    const int h = static_cast<int>(r / pages_b);
    const int64_t page = r - h * pages_b;
    PageRef ref;
    ref.seg = b * p.kv_heads + h;
    ref.page = static_cast<int>(page);
    const int64_t id = load_index(p.block_table, p.table_i64, b * p.table_stride + page);
    ref.id = (id < 0 || id >= p.num_blocks) ? -1 : static_cast<int>(id);
    if (ref.id < 0) report_bad_page_id();
    const int64_t len = p.context_lens ? load_index(p.context_lens, p.lens_i64, b) : p.uniform_len;
    const int64_t left = len - page * kPageTokens;
    ref.meta = static_cast<int>(left < kPageTokens ? left : kPageTokens) |
               ((page == pages_b - 1) ? 0x100 : 0);
    return ref;
}

template <typename T, int D, int NT, int NWARPS, int STAGES>
__global__ void __launch_bounds__(NWARPS * 32)
paged_decode_persistent_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                               const __grid_constant__ CUtensorMap vmap) {
    using Shape = PersistentShape<D, NWARPS, STAGES>;
    using Warp = WarpPageAttention<T, D, NT>;
    constexpr int kGP = 8 * NT;

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[NWARPS][STAGES];
    __shared__ long long warp_sums[NWARPS];

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    int64_t* prefix = reinterpret_cast<int64_t*>(smem + Shape::kStageRegion);
    const uint32_t bar0 = smem_addr(&bars[warp][0]);
    if (lane == 0) {
#pragma unroll
        for (int st = 0; st < STAGES; ++st) mbar_init(bar0 + 8 * st, 1);
    }
    fence_mbar_init();
    wait_for_prior_grid();

    // Pages per sequence and their prefix sums (sequences with no work count 0 pages).
    const int per_thread = (p.batch + blockDim.x - 1) / blockDim.x;
    const int first = threadIdx.x * per_thread;
    long long local = 0;
    for (int k = 0; k < per_thread; ++k) {
        const int b = first + k;
        if (b < p.batch) {
            const SeqSplit s = seq_split(p, b);
            local += s.pages;
        }
    }
    long long incl = local;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const long long v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
    }
    if (lane == 31) warp_sums[warp] = incl;
    __syncthreads();
    long long base = 0;
    for (int v = 0; v < warp; ++v) base += warp_sums[v];
    long long run = base + incl - local;
    for (int k = 0; k < per_thread; ++k) {
        const int b = first + k;
        if (b < p.batch) {
            prefix[b] = run;
            run += seq_split(p, b).pages;
        }
    }
    if (threadIdx.x == blockDim.x - 1) prefix[p.batch] = run;
    __syncthreads();
    allow_next_grid();
    if (blockIdx.x == 0) {
        // The merge pass reads the layout back from the workspace.
        for (int b = threadIdx.x; b <= p.batch; b += blockDim.x) p.prefix_out[b] = prefix[b];
    }

    const int64_t total = static_cast<int64_t>(p.kv_heads) * prefix[p.batch];
    // Never more ranges than pages, so every range in use holds at least one page.
    const int64_t warps = min(static_cast<int64_t>(gridDim.x) * NWARPS, total);
    const int64_t wid = static_cast<int64_t>(blockIdx.x) * NWARPS + warp;
    if (wid >= warps) return;
    const int64_t lo = wid * total / warps;
    const int64_t hi = (wid + 1) * total / warps;
    const int n = static_cast<int>(hi - lo);
    if (n <= 0) return;

    uint8_t* wsm = smem + warp * Shape::kWarpBytes;
    const uint32_t wsm_addr = smem_addr(wsm);

    // Lane j of `cur` describes page 32k + j of the range, `nxt` the next 32.
    PageRef cur, nxt;
    cur.seg = nxt.seg = -1;
    cur.id = nxt.id = -1;
    cur.page = nxt.page = 0;
    cur.meta = nxt.meta = 0;
    if (lane < n) cur = locate_page(p, prefix, lo + lane);
    if (32 + lane < n) nxt = locate_page(p, prefix, lo + 32 + lane);

    auto issue = [&](int i, const PageRef& ref_batch) {
        // Every lane calls this (warp-uniform i): broadcast page i's entry, lane 0 issues.
        const int src = i & 31;
        const int id = __shfl_sync(0xffffffffu, ref_batch.id, src);
        const int seg = __shfl_sync(0xffffffffu, ref_batch.seg, src);
        if (lane == 0) {
            const uint32_t bar = bar0 + 8 * (i % STAGES);
            const uint32_t dst = wsm_addr + (i % STAGES) * Shape::kStageBytes;
            if (id >= 0) {
                const int h = seg % p.kv_heads;
                mbar_arrive_expect_tx(bar, Shape::kStageBytes);
                tma_load_5d(dst, &kmap, 0, 0, 0, h, id, bar);
                tma_load_5d(dst + Shape::kTileBytes, &vmap, 0, 0, 0, h, id, bar);
            } else {
                // No load for a corrupted ID; complete the phase so the ring stays in step.
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
            }
        }
    };

    // L2 prefetch of page j (every lane calls; j within the cur/nxt window).
    auto prefetch = [&](int j, const PageRef& ref_batch) {
        const int src = j & 31;
        const int id = __shfl_sync(0xffffffffu, ref_batch.id, src);
        const int seg = __shfl_sync(0xffffffffu, ref_batch.seg, src);
        if (lane == 0 && id >= 0) {
            const int h = seg % p.kv_heads;
            tma_prefetch_l2_5d(&kmap, 0, 0, 0, h, id);
            tma_prefetch_l2_5d(&vmap, 0, 0, 0, h, id);
        }
    };

    const int prologue = n < STAGES ? n : STAGES;
    for (int i = 0; i < prologue; ++i) issue(i, i < 32 ? cur : nxt);
    for (int i = prologue; kPrefetchPages > 0 && i < n && i < STAGES + kPrefetchPages; ++i)
        prefetch(i, i < 32 ? cur : nxt);

    Warp w;
    int piece_seg = -1;
    int piece_first_page = 0;
    bool piece_bad = false;
    bool first_piece = true;
    bool failed = false;
    float* part_o = p.part_o + wid * 2 * kGP * D;
    float* part_lse = p.part_lse + wid * 2 * kGP;

    for (int i = 0; i < n; ++i) {
        if (i > 0 && (i & 31) == 0) {
            cur = nxt;
            nxt.seg = -1;
            nxt.id = -1;
            if (i + 32 + lane < n) nxt = locate_page(p, prefix, lo + i + 32 + lane);
        }
        const int src = i & 31;
        const int seg = __shfl_sync(0xffffffffu, cur.seg, src);
        const int id = __shfl_sync(0xffffffffu, cur.id, src);
        const int page = __shfl_sync(0xffffffffu, cur.page, src);
        const int meta = __shfl_sync(0xffffffffu, cur.meta, src);
        const int b = seg / p.kv_heads;
        const int h = seg - b * p.kv_heads;
        if (seg != piece_seg) {
            piece_seg = seg;
            piece_first_page = page;
            piece_bad = false;
            w.load_q(p, b, h, lane);
            w.reset();
        }
        const int st = i % STAGES;
        const bool ok = mbar_wait_bounded(bar0 + 8 * st, (i / STAGES) & 1);
        if (!__all_sync(0xffffffffu, ok)) {
            failed = true;
            // Drain loads still in flight (bounded), then stop this warp.
            const int last = i + STAGES < n ? i + STAGES : n;
            for (int j = i + 1; j < last; ++j) mbar_wait_bounded(bar0 + 8 * (j % STAGES), (j / STAGES) & 1);
            if (lane == 0) atomicOr(&g_device_status, kStatusWaitTimeout);
            break;
        }
        const int valid = meta & 0xff;
        typename Warp::PageFrags frags;
        if (id >= 0) {
            const uint32_t kt = wsm_addr + st * Shape::kStageBytes;
            Warp::load_page(frags, kt, kt + Shape::kTileBytes,
                            wsm + st * Shape::kStageBytes + Shape::kTileBytes, valid, lane);
        } else {
            piece_bad = true;
        }

        // The page is in registers: refill its stage before the arithmetic.
        if (i + STAGES < n) {
            fence_proxy_async_smem();  // this lane's shared reads/writes before the TMA write
            __syncwarp();
            const int j = i + STAGES;
            issue(j, (j >> 5) == (i >> 5) ? cur : nxt);
            const int ahead = j + kPrefetchPages;
            if (kPrefetchPages > 0 && ahead < n) prefetch(ahead, (ahead >> 5) == (i >> 5) ? cur : nxt);
        }
        if (id >= 0) w.attend(frags, valid, p.scale_log2, lane);

        // End of a piece: the next page belongs to another segment, or the range ends.
        int next_seg = -1;
        if (i + 1 < n) {
            const int nsrc = (i + 1) & 31;
            next_seg = __shfl_sync(0xffffffffu, ((i + 1) >> 5) == (i >> 5) ? cur.seg : nxt.seg, nsrc);
        }
        if (next_seg != seg) {
            const bool whole = piece_first_page == 0 && (meta & 0x100);
            const int slot = first_piece ? 0 : 1;
            w.reduce_l();
            if (whole) {
                if (piece_bad) {
                    const float nan = __int_as_float(0x7fffffff);
                    T* out = static_cast<T*>(p.out) + b * p.out_stride_seq;
                    for (int idx = lane; idx < p.group * D; idx += 32) {
                        const int g = idx / D;
                        out[static_cast<int64_t>(h * p.group + g) * p.out_stride_head + (idx - g * D)] =
                            from_float<T>(nan);
                    }
                } else {
                    w.store_final(p, b, h, lane);
                }
            } else if (piece_bad) {
                w.store_partial_nan(part_o + slot * kGP * D, part_lse + slot * kGP, p.group, lane);
            } else {
                w.store_partial(part_o + slot * kGP * D, part_lse + slot * kGP, p.group, lane);
            }
            first_piece = false;
        }
    }
    if (failed) {
        // Everything this warp had not finished becomes NaN: cut pieces through
        // both partial slots, whole segments through the output directly.
        const float nan = __int_as_float(0x7fffffff);
        w.store_partial_nan(part_o, part_lse, p.group, lane);
        w.store_partial_nan(part_o + kGP * D, part_lse + kGP, p.group, lane);
        for (int64_t g = lo; g < hi; g += 32) {
            const int64_t mine = g + lane;
            const int seg = mine < hi ? locate_page(p, prefix, mine).seg : -1;
            for (int src = 0; src < 32; ++src) {
                const int s = __shfl_sync(0xffffffffu, seg, src);
                if (s < 0) continue;
                const int b = s / p.kv_heads;
                const int h = s - b * p.kv_heads;
                T* out = static_cast<T*>(p.out) + b * p.out_stride_seq;
                for (int idx = lane; idx < p.group * D; idx += 32) {
                    const int q = idx / D;
                    out[static_cast<int64_t>(h * p.group + q) * p.out_stride_head + (idx - q * D)] =
                        from_float<T>(nan);
                }
            }
        }
    }
}


// ------------------------------------------------------------ cluster kernel
//
// Split-KV without a merge pass: the C split CTAs of one (sequence, KV head)
// segment form a thread-block cluster. Each CTA streams an equal share of the
// segment's pages, combines its warps in shared memory, and leaves its
// normalised partial and log2-sum-exp there; after a cluster barrier every
// CTA reads all C partials through distributed shared memory and writes its
// share of the G x D outputs. No partials go to HBM and nothing waits on
// another grid.

template <int D, int NT, int NWARPS, int STAGES>
struct ClusterShape {
    using Grid = MmaDecodeShape<D, NT, NWARPS, STAGES>;
    static constexpr int kStageRegion = NWARPS * Grid::kWarpBytes;
    static constexpr int kResultBytes = 8 * NT * D * 4;  // this CTA's normalised partial [8*NT][D]
    static constexpr int kSmemBytes = kStageRegion + kResultBytes + 1024;
};

template <typename T, int D, int NT, int NWARPS, int STAGES>
__global__ void __launch_bounds__(NWARPS * 32)
paged_decode_cluster_kernel(const DecodeParams p, const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap) {
    namespace cg = cooperative_groups;
    using Shape = ClusterShape<D, NT, NWARPS, STAGES>;
    using Grid = typename Shape::Grid;
    using Warp = WarpPageAttention<T, D, NT>;
    constexpr int kGP = 8 * NT;

    extern __shared__ uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bars[NWARPS][STAGES];
    __shared__ int warp_flags[NWARPS];
    __shared__ float cta_lse[kGP];  // per query row; -inf: no pages here; NaN: corrupted ID or timeout

    cg::cluster_group cluster = cg::this_cluster();
    const int rank = static_cast<int>(cluster.block_rank());
    const int csize = static_cast<int>(cluster.num_blocks());
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int h = blockIdx.y;
    const int b = blockIdx.z;

    wait_for_prior_grid();
    allow_next_grid();
    const SeqSplit seq = seq_split(p, b);
    if (seq.state != 0) {
        // Every CTA of the cluster takes this branch: none waits on another.
        if (rank == 0) write_group_constant<T>(p, b, h, seq.state == 1 ? 0.0f : __int_as_float(0x7fffffff));
        return;
    }

    uint8_t* smem = reinterpret_cast<uint8_t*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    float* cta_o = reinterpret_cast<float*>(smem + Shape::kStageRegion);
    const int64_t page_begin = seq.pages * rank / csize;
    const int64_t page_end = seq.pages * (rank + 1) / csize;
    const int cta_pages = static_cast<int>(page_end - page_begin);
    const int n_my = warp < cta_pages ? (cta_pages - warp + NWARPS - 1) / NWARPS : 0;

    // Page IDs of this warp's pages, 32 at a time: lane j of `cur` holds page
    // 32k + j of the warp's sequence (run page warp + i * NWARPS), `nxt` the next 32.
    auto load_id = [&](int i) -> long long {
        return i < n_my ? load_index(p.block_table, p.table_i64,
                                     b * p.table_stride + page_begin + warp + static_cast<int64_t>(i) * NWARPS)
                        : 0;
    };
    long long cur = load_id(lane);
    long long nxt = load_id(32 + lane);
    auto id_ok = [&](long long id) { return id >= 0 && id < p.num_blocks; };
    bool warp_bad = false;
    {
        // Whole-warp check of the first batch; later batches are checked as they rotate in.
        warp_bad = __any_sync(0xffffffffu, lane < n_my && !id_ok(cur));
    }
    const uint32_t bar0 = smem_addr(&bars[warp][0]);
    if (lane == 0) {
#pragma unroll
        for (int st = 0; st < STAGES; ++st) mbar_init(bar0 + 8 * st, 1);
    }
    fence_mbar_init();
    __syncwarp();

    uint8_t* wsm = smem + warp * Grid::kWarpBytes;
    const uint32_t wsm_addr = smem_addr(wsm);
    auto issue = [&](int i, long long batch) {
        const long long id = __shfl_sync(0xffffffffu, batch, i & 31);
        if (lane == 0) {
            const int st = i % STAGES;
            const uint32_t bar = bar0 + 8 * st;
            if (id_ok(id)) {
                const uint32_t dst = wsm_addr + st * Grid::kStageBytes;
                mbar_arrive_expect_tx(bar, Grid::kStageBytes);
                tma_load_5d(dst, &kmap, 0, 0, 0, h, static_cast<int>(id), bar);
                tma_load_5d(dst + Grid::kTileBytes, &vmap, 0, 0, 0, h, static_cast<int>(id), bar);
            } else {
                // No load for a corrupted ID; complete the phase so the ring stays in step.
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
            }
        }
    };
    const int prologue = n_my < STAGES ? n_my : STAGES;
    for (int i = 0; i < prologue; ++i) issue(i, cur);

    Warp w;
    w.load_q(p, b, h, lane);
    w.reset();

    bool failed = false;
    int i = 0;
    for (; i < n_my; ++i) {
        if (i > 0 && (i & 31) == 0) {
            cur = nxt;
            nxt = load_id(i + 32 + lane);
            warp_bad |= __any_sync(0xffffffffu, i + lane < n_my && !id_ok(cur));
        }
        const int st = i % STAGES;
        const bool ok = mbar_wait_bounded(bar0 + 8 * st, (i / STAGES) & 1);
        if (!__all_sync(0xffffffffu, ok)) {
            failed = true;
            break;
        }
        const uint32_t kt = wsm_addr + st * Grid::kStageBytes;
        const uint32_t vt = kt + Grid::kTileBytes;
        const int64_t page = page_begin + warp + static_cast<int64_t>(i) * NWARPS;
        const int64_t left = seq.len - page * kPageTokens;
        const int valid = left < kPageTokens ? static_cast<int>(left) : kPageTokens;
        const bool page_ok = id_ok(__shfl_sync(0xffffffffu, cur, i & 31));
        typename Warp::PageFrags frags;
        if (page_ok) Warp::load_page(frags, kt, vt, wsm + st * Grid::kStageBytes + Grid::kTileBytes, valid, lane);
        if (i + STAGES < n_my) {
            fence_proxy_async_smem();  // this lane's shared reads/writes before the TMA write
            __syncwarp();
            const int j = i + STAGES;
            issue(j, (j >> 5) == (i >> 5) ? cur : nxt);
        }
        if (page_ok) w.attend(frags, valid, p.scale_log2, lane);
    }
    if (failed) {
        const int last = i + STAGES < n_my ? i + STAGES : n_my;
        for (int j = i; j < last; ++j) mbar_wait_bounded(bar0 + 8 * (j % STAGES), (j / STAGES) & 1);
        if (lane == 0) atomicOr(&g_device_status, kStatusWaitTimeout);
    }
    if (lane == 0 && warp_bad) report_bad_page_id();
    if (lane == 0) warp_flags[warp] = (failed ? 2 : 0) | (warp_bad ? 1 : 0);
    w.reduce_l();

    // Combine the warps through shared memory (their stages are drained).
    __syncthreads();
    float* red = reinterpret_cast<float*>(wsm);
    float* red_m = red + Grid::kQRows * Grid::kRedStride;
    float* red_l = red_m + Grid::kQRows;
#pragma unroll
    for (int mt = 0; mt < Warp::KS; ++mt) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int d = mt * 16 + (lane >> 2);
            const int q = nt * 8 + 2 * (lane & 3);
            red[q * Grid::kRedStride + d] = w.o[mt][nt][0];
            red[(q + 1) * Grid::kRedStride + d] = w.o[mt][nt][1];
            red[q * Grid::kRedStride + d + 8] = w.o[mt][nt][2];
            red[(q + 1) * Grid::kRedStride + d + 8] = w.o[mt][nt][3];
        }
    }
    if (lane < 4) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int q = nt * 8 + 2 * lane;
            red_m[q] = w.m[nt][0];
            red_m[q + 1] = w.m[nt][1];
            red_l[q] = w.l[nt][0];
            red_l[q + 1] = w.l[nt][1];
        }
    }
    __syncthreads();
    int cta_bad = 0;
#pragma unroll
    for (int v = 0; v < NWARPS; ++v) cta_bad |= warp_flags[v];
    const int G = p.group;
    for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
        const int g = idx / D;
        const int d = idx - g * D;
        float mx = -INFINITY;
#pragma unroll
        for (int v = 0; v < NWARPS; ++v)
            mx = fmaxf(mx, reinterpret_cast<const float*>(smem + v * Grid::kWarpBytes)[Grid::kQRows * Grid::kRedStride + g]);
        float den = 0.0f;
        float num = 0.0f;
#pragma unroll
        for (int v = 0; v < NWARPS; ++v) {
            const float* wr = reinterpret_cast<const float*>(smem + v * Grid::kWarpBytes);
            const float* wm = wr + Grid::kQRows * Grid::kRedStride;
            const float f = mx == -INFINITY ? 0.0f : fast_exp2(wm[g] - mx);
            den += f * wm[Grid::kQRows + g];
            num += f * wr[g * Grid::kRedStride + d];
        }
        cta_o[g * D + d] = den > 0.0f ? num / den : 0.0f;
        if (d == 0)
            cta_lse[g] = cta_bad ? __int_as_float(0x7fffffff) : (den > 0.0f ? mx + log2f(den) : -INFINITY);
    }

    // Every CTA's partial is in its shared memory: combine across the cluster.
    cluster.sync();
    T* out = static_cast<T*>(p.out) + b * p.out_stride_seq;
    const int total = G * D;
    const int begin = total * rank / csize;
    const int end = total * (rank + 1) / csize;
    for (int idx = begin + static_cast<int>(threadIdx.x); idx < end; idx += blockDim.x) {
        const int g = idx / D;
        const int d = idx - g * D;
        float mx = -INFINITY;
        bool nan = false;
        for (int c = 0; c < csize; ++c) {
            const float v = *cluster.map_shared_rank(&cta_lse[g], c);
            nan |= isnan(v);
            mx = fmaxf(mx, v);
        }
        float value = __int_as_float(0x7fffffff);
        if (!nan) {
            float den = 0.0f;
            float num = 0.0f;
            for (int c = 0; c < csize; ++c) {
                const float v = *cluster.map_shared_rank(&cta_lse[g], c);
                const float f = v == -INFINITY ? 0.0f : fast_exp2(v - mx);
                den += f;
                num += f * *cluster.map_shared_rank(&cta_o[g * D + d], c);
            }
            value = num / den;
        }
        out[static_cast<int64_t>(h * G + g) * p.out_stride_head + d] = from_float<T>(value);
    }
    cluster.sync();  // no CTA leaves while another may still read its shared memory
}

}  // namespace mv
