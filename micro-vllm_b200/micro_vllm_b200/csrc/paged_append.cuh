// Paged KV append (reshape-and-cache): scatter new K/V rows into their pages.
//
// Work item = one VEC-byte chunk of one (sequence, token, KV head) row of K or
// V. Consecutive threads take consecutive chunks of a row, so a 128-wide bf16
// row (256 B) is 16 lanes of 16-byte loads and stores; K and V rows of the
// same token are adjacent work items. Bytes move as raw integers: NaN payloads,
// signed zeros and infinities are preserved bit for bit. The destination of
// token t of sequence b is logical position start_b + t, i.e. page
// block_table[b, pos / block_size], slot pos % block_size
// (paged_kv_cache.cu:36-37 in the reference); positions outside the row or
// physical IDs outside the pool are skipped (paged_kv_cache.cu:32-35).
#pragma once

#include "mv_device.cuh"

namespace mv {

constexpr int kAppendThreads = 256;

template <int VEC>
struct VecType;
template <> struct VecType<16> { using type = uint4; };
template <> struct VecType<8> { using type = uint2; };
template <> struct VecType<4> { using type = uint32_t; };
template <> struct VecType<2> { using type = uint16_t; };

template <int VEC>
__global__ void __launch_bounds__(kAppendThreads) write_paged_kv_kernel(const AppendParams a, int64_t total) {
    using V = typename VecType<VEC>::type;
    wait_for_prior_grid();
    allow_next_grid();
    const int chunks = a.row_bytes / VEC;
    const int64_t stride = static_cast<int64_t>(blockDim.x) * gridDim.x;
    for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
         idx += stride) {
        const int chunk = static_cast<int>(idx % chunks);
        const int64_t rest = idx / chunks;
        const int which = static_cast<int>(rest & 1);  // 0 = K, 1 = V
        const int64_t row = rest >> 1;                 // (b * num_tokens + t) * kv_heads + head
        const int head = static_cast<int>(row % a.kv_heads);
        const int64_t bt = row / a.kv_heads;
        const int t = static_cast<int>(bt % a.num_tokens);
        const int b = static_cast<int>(bt / a.num_tokens);

        int64_t start = a.start;
        if (a.positions) {
            start = load_index(a.positions, a.positions_i64, b);
            if (a.positions_end) start -= a.num_tokens;
        }
        const int64_t pos = start + t;
        if (pos < 0) continue;
        const int64_t logical = pos / a.block_size;
        if (logical >= a.blocks_per_seq) continue;
        const int64_t phys = load_index(a.block_table, a.table_i64, b * a.table_stride + logical);
        if (phys < 0 || phys >= a.num_blocks) {
            report_bad_page_id();
            continue;
        }

        const int64_t* sstr = which ? a.value_stride : a.key_stride;
        const uint8_t* src = static_cast<const uint8_t*>(which ? a.value : a.key) +
                             (b * sstr[0] + head * sstr[1] + t * sstr[2]) * a.elem_bytes +
                             static_cast<int64_t>(chunk) * VEC;
        uint8_t* dst = static_cast<uint8_t*>(which ? a.v_cache : a.k_cache) +
                       ((phys * a.kv_heads + head) * a.block_size + (pos - logical * a.block_size)) *
                           static_cast<int64_t>(a.row_bytes) +
                       static_cast<int64_t>(chunk) * VEC;
        *reinterpret_cast<V*>(dst) = *reinterpret_cast<const V*>(src);
    }
}

}  // namespace mv
