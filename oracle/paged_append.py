"""Bit-exact restatement of the paged KV append (test infrastructure only).

Follows ``PagedKVCache._append_cpu`` (src/micro_vllm/paged_kv_cache.py:151-161):
token ``t`` of a chunk that starts at logical position ``start`` lands in
logical page ``(start+t) // page_size``, slot ``(start+t) % page_size`` of the
physical page the table names. The native kernel additionally skips writes
whose physical ID falls outside the pool instead of touching memory
(src/micro_vllm/csrc/paged_kv_cache.cu:32-35); that guard is restated here so
the oracle also covers corrupted tables.

Batched form: the reference holds one request per cache, so a batch is B
caches sharing one pool, each with its own table row and start. Positions past
the row's ``blocks_per_seq`` logical pages, and negative positions, are
skipped -- the device kernel's bounds contract for a device-side start that
the host cannot validate.
"""
import numpy as np


def _as_bits(array: np.ndarray) -> np.ndarray:
    """Reinterpret a float array as unsigned integers of the same width."""
    kind = {2: np.uint16, 4: np.uint32, 8: np.uint64}[array.dtype.itemsize]
    return array.view(kind)


def append_tokens(key_pool, value_pool, key, value, block_table, starts,
                  blocks_per_seq=None):
    """Write ``key``/``value`` [B, Hkv, N, D] into pools [P, Hkv, bs, D] in place.

    ``block_table`` is [B, max_pages] (int32 or int64), ``starts`` is [B] (the
    logical position of each sequence's first new token). Copies move raw
    bits, so NaN payloads, signed zeros and infinities survive exactly, as
    the reference test test/test_cuda_paged_cache.py:78-93 requires.
    """
    key_pool = np.asarray(key_pool)
    value_pool = np.asarray(value_pool)
    num_pages, heads, page_size, dim = key_pool.shape
    batch, src_heads, tokens, src_dim = key.shape
    if (src_heads, src_dim) != (heads, dim) or value.shape != key.shape:
        raise ValueError('K/V shape must match [B, Hkv, N, D] of the pool')
    table = np.asarray(block_table).reshape(batch, -1).astype(np.int64)
    if blocks_per_seq is None:
        blocks_per_seq = table.shape[1]
    starts = np.asarray(starts, dtype=np.int64).reshape(batch)
    positions = starts[:, None] + np.arange(tokens, dtype=np.int64)[None, :]
    logical = np.floor_divide(positions, page_size)
    slot = positions - logical * page_size
    in_row = (positions >= 0) & (logical < blocks_per_seq)
    safe_logical = np.where(in_row, logical, 0)
    physical = np.take_along_axis(table, safe_logical, axis=1)
    valid = in_row & (physical >= 0) & (physical < num_pages)
    seq_idx, tok_idx = np.nonzero(valid)
    phys = physical[seq_idx, tok_idx]
    slots = slot[seq_idx, tok_idx]
    for pool, source in ((key_pool, key), (value_pool, value)):
        pool_bits = _as_bits(pool)
        src_bits = _as_bits(np.ascontiguousarray(source))
        # [n_valid, Hkv, D] rows, written in (sequence, token) order like the CPU loop.
        pool_bits[phys, :, slots, :] = src_bits[seq_idx, :, tok_idx, :]
    return key_pool, value_pool
