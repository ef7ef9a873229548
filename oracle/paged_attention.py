"""Paged GQA decode attention restated on the CPU (test infrastructure only).

Three forms, all over the same paged layout: K/V pools [P, Hkv, bs, D], a
block table [B, max_pages], context lengths [B] (each including the token
appended this step) and queries [B, Hq, D]. Arrays use the storage
representations of ``oracle.dtypes`` (bf16 as uint16 bits).

* ``decode_reference`` -- the reference CPU path, including where it rounds to
  the input dtype: gather pages in logical order (paged_kv_cache.py:178-193),
  fold each GQA group into query rows, ``scores = q @ k^T`` in the input dtype
  then ``.mul_(D ** -0.5)`` (attention.py:85-87), fp32 softmax, probabilities
  cast back to the input dtype (attention.py:91), ``P @ V`` in the input dtype
  (attention.py:93). Used to pin the oracle against the reference's outputs.
* ``decode_float`` -- the same mathematics on inputs widened to float32/64
  with no intermediate rounding: the parity oracle for the GPU kernels
  (the fp32 reference on upcast inputs for bf16).
* ``decode_fp64_per_head`` -- the per-head fp64 loop of
  test/test_cuda_gqa.py:14-23, used for precision known-answer cases.

Edge contract (the GPU kernels follow the same one): a used logical page whose
physical ID lies outside the pool makes that sequence's whole GQA group NaN,
as the reference kernel does (decode_attention_paged.cu:30-37 with
online_attention.cuh:129-134). A context length of 0 yields zeros; a negative
length or one beyond the table row's capacity yields NaN. The reference
rejects those lengths on the host (decode_attention.cpp:98-99); a batched call
carries lengths on the device where the host cannot see them.
"""
import numpy as np

from .dtypes import from_float32, to_float32, round_through


def gather_sequence(pool: np.ndarray, table_row: np.ndarray, length: int) -> np.ndarray:
    """Logical-order copy [Hkv, length, D] of one sequence's pages.

    Restates ``PagedKVCache._gather_buffer`` (paged_kv_cache.py:172-180): take
    ``min(page_size, remaining)`` slots from each used page, concatenate on
    the token axis.
    """
    num_pages, heads, page_size, dim = pool.shape
    used = -(-length // page_size)
    ids = np.asarray(table_row[:used], dtype=np.int64)
    pages = pool[ids]                      # [used, Hkv, bs, D]
    seq = pages.transpose(1, 0, 2, 3).reshape(heads, used * page_size, dim)
    return seq[:, :length]


def _sequence_status(table_row, length, num_pages, page_size, blocks_per_seq):
    """'ok', 'empty' (length 0) or 'nan' (invalid length or page ID)."""
    if length == 0:
        return 'empty'
    if length < 0 or length > blocks_per_seq * page_size:
        return 'nan'
    used = -(-length // page_size)
    ids = np.asarray(table_row[:used], dtype=np.int64)
    if ((ids < 0) | (ids >= num_pages)).any():
        return 'nan'
    return 'ok'


def _group_query(q_row: np.ndarray, kv_heads: int) -> np.ndarray:
    q_heads, dim = q_row.shape
    return q_row.reshape(kv_heads, q_heads // kv_heads, dim)


def _softmax(scores: np.ndarray) -> np.ndarray:
    shifted = scores - scores.max(axis=-1, keepdims=True)
    weights = np.exp(shifted)
    return weights / weights.sum(axis=-1, keepdims=True)


def decode_reference(q, key_pool, value_pool, block_table, context_lens, dtype):
    """The reference CPU path with its dtype roundings; returns storage dtype [B, Hq, D].

    Scale is ``D ** -0.5`` because attention.py:87 fixes it.
    """
    q = np.asarray(q)
    batch, q_heads, dim = q.shape
    num_pages, kv_heads, page_size, _ = key_pool.shape
    table = np.asarray(block_table).reshape(batch, -1)
    scale = dim ** -0.5
    out = np.empty((batch, q_heads, dim), dtype=np.float32)
    for b in range(batch):
        length = int(context_lens[b])
        k = to_float32(gather_sequence(key_pool, table[b], length), dtype).astype(np.float64)
        v = to_float32(gather_sequence(value_pool, table[b], length), dtype).astype(np.float64)
        qg = _group_query(to_float32(q[b], dtype), kv_heads).astype(np.float64)
        # torch.matmul in the input dtype accumulates wider and rounds once.
        scores = round_through((qg @ k.transpose(0, 2, 1)).astype(np.float32), dtype)
        scores = round_through((scores.astype(np.float64) * scale).astype(np.float32), dtype)
        probs = _softmax(scores.astype(np.float32)).astype(np.float32)
        probs = round_through(probs, dtype).astype(np.float64)
        result = round_through((probs @ v).astype(np.float32), dtype)
        out[b] = result.reshape(q_heads, dim)
    return from_float32(out, dtype)


def decode_float(q, key_pool, value_pool, block_table, context_lens, scale, dtype,
                 accum=np.float64, blocks_per_seq=None):
    """Softmax(q K^T * scale) V on widened inputs; returns ``accum`` [B, Hq, D]."""
    q = np.asarray(q)
    batch, q_heads, dim = q.shape
    num_pages, kv_heads, page_size, _ = key_pool.shape
    table = np.asarray(block_table).reshape(batch, -1)
    if blocks_per_seq is None:
        blocks_per_seq = table.shape[1]
    out = np.zeros((batch, q_heads, dim), dtype=accum)
    for b in range(batch):
        length = int(context_lens[b])
        status = _sequence_status(table[b], length, num_pages, page_size, blocks_per_seq)
        if status == 'empty':
            continue
        if status == 'nan':
            out[b] = np.nan
            continue
        k = to_float32(gather_sequence(key_pool, table[b], length), dtype).astype(accum)
        v = to_float32(gather_sequence(value_pool, table[b], length), dtype).astype(accum)
        qg = _group_query(to_float32(q[b], dtype), kv_heads).astype(accum)
        scores = (qg @ k.transpose(0, 2, 1)) * accum(scale)
        out[b] = (_softmax(scores) @ v).reshape(q_heads, dim)
    return out


def decode_fp64_per_head(q, key, value):
    """Per-head fp64 loop of test/test_cuda_gqa.py:14-23.

    ``q`` [Hq, D], contiguous ``key``/``value`` [Hkv, L, D] as float arrays;
    returns float64 [Hq, D]. Scale is ``D ** -0.5``.
    """
    q = np.asarray(q, dtype=np.float64)
    key = np.asarray(key, dtype=np.float64)
    value = np.asarray(value, dtype=np.float64)
    q_heads, dim = q.shape
    group = q_heads // key.shape[0]
    out = np.empty((q_heads, dim), dtype=np.float64)
    for head in range(q_heads):
        kv = head // group
        scores = key[kv] @ q[head] * dim ** -0.5
        weights = np.exp(scores - scores.max())
        out[head] = (weights / weights.sum()) @ value[kv]
    return out
