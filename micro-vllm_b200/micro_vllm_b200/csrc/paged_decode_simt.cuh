// Paged GQA decode on CUDA cores, for every shape the tensor-core kernel does
// not take: fp32, odd head_dim (33, 257, ...), page sizes other than 16, GQA
// groups above 16, unaligned caches.
//
// Same work split as the tensor-core kernel -- one CTA per (split, KV head,
// sequence), so each K/V element is read from HBM once for the whole GQA
// group -- and the same partial-output format for the merge kernel. Tokens
// are processed in 32-token tiles staged in shared memory (fp32), with coalesced
// row loads that follow the page table. The online softmax keeps the
// normalised running output u/l exactly as the reference kernel does
// (online_attention.cuh:47-89): each tile rescales the old output by
// old_mass / new_denominator and adds its weights already divided by the new
// denominator, so large finite V (+-2e38 in fp32) cannot overflow the state.
#pragma once

#include "mv_device.cuh"

namespace mv {

constexpr int kSimtThreads = 128;
constexpr int kSimtLoads = 8;   // K/V tile elements each thread has in flight
constexpr int kSimtTile = 32;  // tokens per tile == warp width (one lane per token)

// Shared-memory floats the SIMT kernel needs (+ token offsets as int64).
__host__ __device__ inline size_t simt_smem_bytes(int group, int head_dim) {
    const size_t row = static_cast<size_t>(head_dim) + 1;  // padded: conflict-free column reads
    const size_t floats = group * row                      // q
                          + 2 * kSimtTile * row            // K and V tile
                          + group * kSimtTile              // scores, then weights
                          + static_cast<size_t>(group) * head_dim  // running output
                          + 3 * static_cast<size_t>(group);         // m, l, rescale
    return ((floats * 4 + 15) / 16) * 16 + 2 * kSimtTile * sizeof(int64_t);
}

template <typename T>
__global__ void __launch_bounds__(kSimtThreads) paged_decode_simt_kernel(const DecodeParams p) {
    extern __shared__ __align__(16) float sm[];
    __shared__ int cta_bad;
    const int G = p.group;
    const int D = p.head_dim;
    const int DP = D + 1;
    const int bs = p.block_size;
    float* q_s = sm;
    float* k_s = q_s + G * DP;
    float* v_s = k_s + kSimtTile * DP;
    float* p_s = v_s + kSimtTile * DP;
    float* acc = p_s + G * kSimtTile;
    float* m_s = acc + G * D;
    float* l_s = m_s + G;
    float* r_s = l_s + G;
    int64_t* off_s = reinterpret_cast<int64_t*>(
        reinterpret_cast<uint8_t*>(sm) + simt_smem_bytes(G, D) - 2 * kSimtTile * sizeof(int64_t));
    int64_t* voff_s = off_s + kSimtTile;  // V offsets (contiguous caches; paged K and V share offsets)

    const int tid = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;
    const int split = blockIdx.x;
    const int h = blockIdx.y;
    const int b = blockIdx.z;

    wait_for_prior_grid();
    allow_next_grid();
    const SeqSplit seq = seq_split(p, b);
    if (split >= seq.splits) return;
    if (seq.state != 0) {
        if (p.new_key) append_row_elements<T>(p, b, h, seq.len);
        write_group_constant<T>(p, b, h, seq.state == 1 ? 0.0f : __int_as_float(0x7fffffff));
        return;
    }
    const bool single = seq.splits == 1;
    // Fused RoPE without a table row for the step's position: NaN, no append.
    const bool rope_missing = p.rope_cos && seq.len - 1 >= p.rope_rows;
    int64_t page_begin, page_end;
    split_range(p, seq, split, &page_begin, &page_end);

    if (tid == 0) cta_bad = rope_missing ? 1 : 0;
    __syncthreads();
    const int64_t seq_row = row_seq(p, b);  // the sequence this query row belongs to
    for (int64_t pg = page_begin + tid; !p.contiguous && pg < page_end; pg += blockDim.x) {
        const int64_t id = load_index(p.block_table, p.table_i64, seq_row * p.table_stride + pg);
        if (id < 0 || id >= p.num_blocks) {
            atomicOr(&cta_bad, 1);
            report_bad_page_id();
        }
    }
    __syncthreads();
    if (cta_bad) {
        // The fused append still writes the new row when its own page is valid,
        // exactly as the append kernel would (a position without a RoPE table row
        // is skipped inside).
        if (p.new_key && split == seq.splits - 1) append_row_elements<T>(p, b, h, seq.len);
        if (single) write_group_constant<T>(p, b, h, __int_as_float(0x7fffffff));
        else write_group_partial_nan(p, b, h, split);
        return;
    }

    const T* q = static_cast<const T*>(p.q) + row_q_offset(p, b);
    for (int idx = tid; idx < G * D; idx += blockDim.x) {
        const int g = idx / D;
        const int d = idx - g * D;
        q_s[g * DP + d] = to_float<T>(q[static_cast<int64_t>(h * G + g) * p.q_stride_head + d]);
        acc[idx] = 0.0f;
    }
    for (int g = tid; g < G; g += blockDim.x) {
        m_s[g] = -INFINITY;
        l_s[g] = 0.0f;
    }
    if (p.rope_cos) {
        // Rotate the staged query rows at the step's position, pair (d, d + D/2) per thread.
        __syncthreads();
        const int half = D / 2;
        const int64_t pos = seq.len - 1;
        const T* cs = static_cast<const T*>(p.rope_cos) + pos * D;
        const T* sn = static_cast<const T*>(p.rope_sin) + pos * D;
        for (int idx = tid; idx < G * half; idx += blockDim.x) {
            const int g = idx / half;
            const int d = idx - g * half;
            float* row = q_s + g * DP;
            const float x0 = row[d], x1 = row[d + half];
            row[d] = rope_element<T>(x0, x1, to_float<T>(cs[d]), to_float<T>(sn[d]), true);
            row[d + half] = rope_element<T>(x1, x0, to_float<T>(cs[d + half]), to_float<T>(sn[d + half]), false);
        }
    }
    // Fused append: this split holds the step's new token (position len - 1)
    // when it holds the sequence's last page.
    const int64_t new_tok = (p.new_key && split == seq.splits - 1) ? seq.len - 1 : -1;

    const T* kc = static_cast<const T*>(p.k_cache);
    const T* vc = static_cast<const T*>(p.v_cache);
    const int64_t tok_begin = page_begin * bs;
    const int64_t tok_end_raw = page_end * bs;
    const int64_t tok_end = tok_end_raw < seq.len ? tok_end_raw : seq.len;

    for (int64_t t0 = tok_begin; t0 < tok_end; t0 += kSimtTile) {
        const int count = static_cast<int>(tok_end - t0 < kSimtTile ? tok_end - t0 : kSimtTile);
        if (tid < count) {
            const int64_t tok = t0 + tid;
            if (p.contiguous) {
                off_s[tid] = seq_row * p.k_stride[0] + h * p.k_stride[1] + tok * p.k_stride[2];
                voff_s[tid] = seq_row * p.v_stride[0] + h * p.v_stride[1] + tok * p.v_stride[2];
            } else {
                const int64_t pg = tok / bs;
                const int64_t id = load_index(p.block_table, p.table_i64, seq_row * p.table_stride + pg);
                off_s[tid] = voff_s[tid] = ((id * p.kv_heads + h) * bs + (tok - pg * bs)) * D;
            }
        }
        __syncthreads();
        // kSimtLoads elements of K and V per thread in flight at once (loads
        // first, then the shared-memory stores), not one round trip each.
        for (int base = 0; base < count * D; base += kSimtThreads * kSimtLoads) {
            float kv[kSimtLoads], vv[kSimtLoads];
#pragma unroll
            for (int u = 0; u < kSimtLoads; ++u) {
                const int idx = base + u * kSimtThreads + tid;
                if (idx < count * D) {
                    const int t = idx / D;
                    const int d = idx - t * D;
                    kv[u] = to_float<T>(kc[off_s[t] + d]);
                    vv[u] = to_float<T>(vc[voff_s[t] + d]);
                }
            }
#pragma unroll
            for (int u = 0; u < kSimtLoads; ++u) {
                const int idx = base + u * kSimtThreads + tid;
                if (idx < count * D) {
                    const int t = idx / D;
                    const int d = idx - t * D;
                    k_s[t * DP + d] = kv[u];
                    v_s[t * DP + d] = vv[u];
                }
            }
        }
        __syncthreads();
        if (new_tok >= t0 && new_tok < t0 + count) {
            // The tile's old row of the new token is read (by every thread, above):
            // replace it in shared memory and in the pool with the new K/V row.
            using Raw = typename std::conditional<sizeof(T) == 2, uint16_t, uint32_t>::type;
            const int r = static_cast<int>(new_tok - t0);
            const T* krow = static_cast<const T*>(p.new_key) + b * p.new_key_stride[0] + h * p.new_key_stride[1];
            const T* vrow = static_cast<const T*>(p.new_value) + b * p.new_value_stride[0] + h * p.new_value_stride[1];
            const int half = D / 2;
            for (int d = tid; d < D; d += blockDim.x) {
                T kval = krow[d];
                if (p.rope_cos) {
                    const bool first = d < half;
                    kval = from_float<T>(rope_element<T>(
                        to_float<T>(krow[d]), to_float<T>(krow[first ? d + half : d - half]),
                        to_float<T>(static_cast<const T*>(p.rope_cos)[new_tok * D + d]),
                        to_float<T>(static_cast<const T*>(p.rope_sin)[new_tok * D + d]), first));
                }
                k_s[r * DP + d] = to_float<T>(kval);
                v_s[r * DP + d] = to_float<T>(vrow[d]);
                // The pool rows are written through the decode's const pointers (the caller's writable pools).
                Raw* kpool = const_cast<Raw*>(static_cast<const Raw*>(p.k_cache));
                Raw* vpool = const_cast<Raw*>(static_cast<const Raw*>(p.v_cache));
                kpool[off_s[r] + d] = p.rope_cos ? *reinterpret_cast<const Raw*>(&kval)
                                                 : reinterpret_cast<const Raw*>(krow)[d];
                vpool[voff_s[r] + d] = reinterpret_cast<const Raw*>(vrow)[d];
            }
            __syncthreads();
        }
        for (int idx = tid; idx < G * kSimtTile; idx += blockDim.x) {
            const int g = idx / kSimtTile;
            const int t = idx - g * kSimtTile;
            float s = -INFINITY;
            if (t < count) {
                const float* qr = q_s + g * DP;
                const float* kr = k_s + t * DP;
                // Four independent partial sums: the shared-memory loads and FMAs pipeline.
                float d0 = 0.0f, d1 = 0.0f, d2 = 0.0f, d3 = 0.0f;
                int d = 0;
                for (; d + 3 < D; d += 4) {
                    d0 = fmaf(qr[d], kr[d], d0);
                    d1 = fmaf(qr[d + 1], kr[d + 1], d1);
                    d2 = fmaf(qr[d + 2], kr[d + 2], d2);
                    d3 = fmaf(qr[d + 3], kr[d + 3], d3);
                }
                for (; d < D; ++d) d0 = fmaf(qr[d], kr[d], d0);
                s = ((d0 + d1) + (d2 + d3)) * p.scale_log2;
            }
            p_s[idx] = s;
        }
        __syncthreads();
        for (int g = warp; g < G; g += kSimtThreads / 32) {
            const float s = p_s[g * kSimtTile + lane];
            const float m_old = m_s[g];
            const float m_new = fmaxf(m_old, warp_max(s));
            const float e = fast_exp2(s - m_new);
            const float tile_mass = warp_sum(e);
            const float old_mass = m_old == -INFINITY ? 0.0f : fast_exp2(m_old - m_new) * l_s[g];
            const float l_new = old_mass + tile_mass;
            p_s[g * kSimtTile + lane] = e / l_new;
            __syncwarp();
            if (lane == 0) {
                m_s[g] = m_new;
                l_s[g] = l_new;
                r_s[g] = old_mass / l_new;
            }
        }
        __syncthreads();
        for (int idx = tid; idx < G * D; idx += blockDim.x) {
            const int g = idx / D;
            const int d = idx - g * D;
            const float* w = p_s + g * kSimtTile;
            float a = acc[idx] * r_s[g];
            for (int t = 0; t < count; ++t) a = fmaf(w[t], v_s[t * DP + d], a);
            acc[idx] = a;
        }
        __syncthreads();
    }

    T* out = static_cast<T*>(p.out);
    for (int idx = tid; idx < G * D; idx += blockDim.x) {
        const int g = idx / D;
        const int d = idx - g * D;
        if (single) {
            out[row_out_offset(p, b) + static_cast<int64_t>(h * G + g) * p.out_stride_head + d] =
                from_float<T>(acc[idx]);
        } else {
            const int64_t row = (static_cast<int64_t>(b) * p.q_heads + h * G + g) * p.max_splits + split;
            p.part_o[row * D + d] = acc[idx];
            if (d == 0) p.part_lse[row] = m_s[g] + log2f(l_s[g]);
        }
    }
}

}  // namespace mv
