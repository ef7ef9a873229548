"""Paged GQA decode attention: drop-in for the paged path of ``micro_vllm.cuda_attention``.

Reference-shaped API (same names, arguments, error types and messages):

* ``decode_attention_paged(query, cache, *, layer_idx)`` --
  src/micro_vllm/cuda_attention.py:116-135 with ``_checked_paged_query``
  (:86-113). Accepts the reference's own ``PagedKVCache`` and reads its
  pages in place.
* ``_load_extension()._decode_attention_paged(query, key_pages, value_pages,
  table, length)`` -- the native entry point and its metadata checks
  (src/micro_vllm/csrc/decode_attention.cpp:17-124, 147-152).

Batched API (new surface; the reference is batch 1):

* ``paged_decode_attention(query, key_cache, value_cache, block_table,
  context_lens, scale)`` over one shared page pool, with bf16 support.

All of them run libmvdecode.so's sm_100a kernels through the C ABI
(``mv_paged_decode``): the TMA + tensor-core split-KV kernel for fp16/bf16
with block size 16 and head_dim 64/128/256, the CUDA-core split-KV kernel for
every other shape (fp32, odd head_dim or page size). Importing this module
loads nothing; there is no CPU path.
"""
import ctypes
from functools import lru_cache

import torch

from . import _native
from ._tensors import DTYPE_CODES, INDEX_CODES, current_stream_handle, current_stream_raw

_INT64_MAX = 2 ** 63 - 1


def _check(condition, message):
    if not condition:
        raise RuntimeError(message)


def _validate_storage(tensor):
    _check(tensor.is_cuda, 'decode_attention requires CUDA tensors')
    _check(tensor.layout == torch.strided, 'decode_attention requires strided tensors')
    _check(not tensor.requires_grad, 'decode_attention does not support gradients')
    _check(not tensor.is_neg(), 'decode_attention does not support lazy negative views')


def _validate_gqa_tensor(tensor):
    _validate_storage(tensor)
    _check(tensor.dtype in (torch.float32, torch.float16), 'GQA requires float32 or float16 tensors')


def _validate_gqa_strides(tensor):
    _check(tensor.stride(3) == 1, 'GQA requires feature stride 1')
    _check(all(tensor.stride(d) >= 0 for d in range(3)), 'GQA requires nonnegative outer strides')


def _validate_gqa_inputs(query, key, value):
    """decode_attention.cpp:61-82, same order and messages."""
    for tensor in (query, key, value):
        _validate_gqa_tensor(tensor)
    _check(query.dtype == key.dtype == value.dtype, 'Q, K, V must use the same dtype')
    _check(query.device == key.device == value.device, 'Q, K, V must use the same device')
    _check(query.dim() == 4 and key.dim() == 4 and value.dim() == 4,
           'Q must have shape [1,Hq,1,D] and K/V must have shape [1,Hkv,L,D]')
    for tensor in (query, key, value):
        _validate_gqa_strides(tensor)
    _check(query.shape[0] == 1 and key.shape[0] == 1 and value.shape[0] == 1,
           'GQA currently requires batch size 1')
    _check(query.numel() > 0 and key.numel() > 0 and value.numel() > 0,
           'head counts, context length, and head dimension must be positive')
    _check(query.shape[2] == 1, 'GQA decode requires exactly one query token')
    _check(key.shape == value.shape, 'K and V must have the same shape')
    _check(query.shape[3] == key.shape[3], 'Q and K/V must share the head dimension')
    _check(query.shape[1] % key.shape[1] == 0, 'query head count must be divisible by KV head count')


def _validate_paged_table(table, key, query, length):
    _validate_storage(table)
    _check(table.dtype == torch.int64, 'page table requires int64')
    _check(table.dim() == 1, 'page table must be one-dimensional')
    _check(table.is_contiguous(), 'page table must be contiguous')
    _check(table.device == query.device, 'Q, K/V pages and table must use the same device')
    _check(table.shape[0] > 0, 'page table length must be positive')
    _check(table.shape[0] <= key.shape[0], 'page table length exceeds physical pages')
    _check(table.shape[0] <= _INT64_MAX // key.shape[2], 'page table capacity exceeds int64 bounds')
    _check(length > 0, 'context length must be positive')
    _check(length <= table.shape[0] * key.shape[2], 'context length exceeds page table capacity')


def _validate_paged_inputs(query, key, value, table, length):
    for tensor in (query, key, value):
        _validate_gqa_tensor(tensor)
    _check(query.dtype == key.dtype == value.dtype, 'Q and K/V pages must use the same dtype')
    _check(query.device == key.device == value.device, 'Q and K/V pages must use the same device')
    _check(query.dim() == 4 and key.dim() == 4 and value.dim() == 4,
           'Q must have shape [1,Hq,1,D] and K/V pages shape [P,Hkv,B,D]')
    _validate_gqa_strides(query)
    _check(key.is_contiguous() and value.is_contiguous(), 'K/V pages must be contiguous')
    _check(query.shape[0] == 1, 'paged attention requires batch size 1')
    _check(query.numel() > 0 and key.numel() > 0 and value.numel() > 0,
           'page dimensions, head counts, and head dimension must be positive')
    _check(query.shape[2] == 1, 'paged decode requires exactly one query token')
    _check(key.shape == value.shape, 'K and V pages must have the same shape')
    _check(query.shape[3] == key.shape[3], 'Q and K/V pages must share the head dimension')
    _check(query.shape[1] % key.shape[1] == 0, 'query head count must be divisible by KV head count')
    _validate_paged_table(table, key, query, length)


# Split-KV scratch per (device, stream): its arrival counters must be zero before
# first use and every completed call leaves them zero, so buffers are zeroed once
# and reused by the calls ordered on that stream.
_WORKSPACES = {}
# Buffers a larger one replaced. A CUDA graph that captured a call keeps that
# call's workspace address, so a buffer once handed to the library is never
# freed while the process runs: freeing it would leave the graph writing into
# memory the allocator may give to others or release (torch.cuda.graph empties
# the allocator's cache when a capture starts).
_RETIRED_WORKSPACES = []


def _workspace(device, stream, nbytes):
    key = (device.index, stream)
    cached = _WORKSPACES.get(key)
    if cached is not None and cached.numel() >= nbytes:
        return cached
    buffer = torch.zeros(nbytes, dtype=torch.uint8, device=device)
    if not torch.cuda.is_current_stream_capturing():
        if cached is not None:
            _RETIRED_WORKSPACES.append(cached)
        _WORKSPACES[key] = buffer
    return buffer


def _run(query3, q_strides, key_cache, value_cache, block_table, table_stride, blocks_per_seq,
         context_lens, max_context_len, scale, out, out_strides, pages_per_split=0, flags=0,
         rows=None):
    """Plan, allocate the split-KV workspace, and launch ``mv_paged_decode``
    (``mv_paged_decode_append`` when ``rows`` holds this step's new K/V rows)."""
    lib = _native.library()
    batch, q_heads, dim = query3
    num_blocks, kv_heads, block_size, _ = key_cache.shape
    dtype = DTYPE_CODES[key_cache.dtype]
    device = key_cache.device
    with torch.cuda.device(device):
        size = ctypes.c_size_t(0)
        _native.check(lib.mv_paged_decode_workspace_size(
            batch, q_heads, kv_heads, dim, block_size, max_context_len, pages_per_split, flags,
            dtype, ctypes.byref(size)))
        stream = current_stream_handle(device)
        workspace = _workspace(device, stream, size.value) if size.value else None
        head = (out.q_ptr, q_strides[0], q_strides[1])
        if rows is not None:
            new_key, new_value, tables = rows
            head += (new_key.data_ptr(), new_key.stride(0), new_key.stride(1),
                     new_value.data_ptr(), new_value.stride(0), new_value.stride(1))
            head += ((tables[0].data_ptr(), tables[1].data_ptr(), tables[0].shape[0]) if tables is not None
                     else (None, None, 0))
        entry = lib.mv_paged_decode if rows is None else lib.mv_paged_decode_append
        _native.check(entry(
            *head,
            key_cache.data_ptr(), value_cache.data_ptr(), num_blocks,
            kv_heads, block_size, dim,
            block_table.data_ptr(), INDEX_CODES[block_table.dtype], table_stride, blocks_per_seq,
            context_lens.data_ptr() if context_lens is not None else None,
            INDEX_CODES[context_lens.dtype] if context_lens is not None else 0,
            max_context_len, batch, q_heads, float(scale),
            out.out_ptr, out_strides[0], out_strides[1],
            workspace.data_ptr() if workspace is not None else None,
            workspace.numel() if workspace is not None else 0,
            pages_per_split, flags, dtype, stream))


def _run_contiguous(q3, q_strides, key, value, context_lens, bound, scale, out, out_strides,
                    pages_per_split=0, flags=0):
    """Plan, allocate the split-KV workspace, and launch ``mv_contiguous_decode``.
    key/value: [B, Hkv, L, D] views (any nonnegative outer strides)."""
    lib = _native.library()
    batch, q_heads, dim = q3
    kv_heads, cache_len = key.shape[1], key.shape[2]
    dtype = DTYPE_CODES[key.dtype]
    device = key.device
    ks = (key.stride(0), key.stride(1), key.stride(2))
    vs = (value.stride(0), value.stride(1), value.stride(2))
    with torch.cuda.device(device):
        path, pps, splits = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        size = ctypes.c_size_t(0)
        _native.check(lib.mv_contiguous_decode_plan(
            key.data_ptr(), *ks, value.data_ptr(), *vs, cache_len, kv_heads, dim, bound, batch, q_heads,
            pages_per_split, flags, dtype, ctypes.byref(path), ctypes.byref(pps), ctypes.byref(splits),
            ctypes.byref(size)))
        stream = current_stream_handle(device)
        workspace = _workspace(device, stream, size.value) if size.value else None
        _native.check(lib.mv_contiguous_decode(
            out.q_ptr, q_strides[0], q_strides[1], key.data_ptr(), *ks, value.data_ptr(), *vs, cache_len,
            kv_heads, dim, context_lens.data_ptr() if context_lens is not None else None,
            INDEX_CODES[context_lens.dtype] if context_lens is not None else 0, bound, batch, q_heads,
            float(scale), out.out_ptr, out_strides[0], out_strides[1],
            workspace.data_ptr() if workspace is not None else None,
            workspace.numel() if workspace is not None else 0, pages_per_split, flags, dtype, stream))
    return _native.PATH_NAMES[path.value], pps.value, splits.value


class _Pointers:
    __slots__ = ('q_ptr', 'out_ptr')

    def __init__(self, q_ptr, out_ptr):
        self.q_ptr = q_ptr
        self.out_ptr = out_ptr


class _DecodeAttentionExtension:
    """The object ``_load_extension()`` returns, shaped like the reference's pybind module."""

    def decode_attention_gqa(self, query, key, value):
        """Q [1,Hq,1,D] over contiguous K/V [1,Hkv,L,D] (any nonnegative outer strides); fresh output."""
        _validate_gqa_inputs(query, key, value)
        output = torch.empty(query.shape, dtype=query.dtype, device=query.device)
        _run_contiguous((1, query.shape[1], query.shape[3]), (0, query.stride(1)), key, value, None,
                        key.shape[2], query.shape[3] ** -0.5, _Pointers(query.data_ptr(), output.data_ptr()),
                        (0, output.stride(1)))
        return output

    def _decode_attention_paged(self, query, key_pages, value_pages, table, length):
        """Internal paged decode for Q [1,Hq,1,D] over pages [P,Hkv,B,D]; fresh output."""
        _validate_paged_inputs(query, key_pages, value_pages, table, length)
        output = torch.empty(query.shape, dtype=query.dtype, device=query.device)
        _run((1, query.shape[1], query.shape[3]), (0, query.stride(1)), key_pages, value_pages,
             table, table.numel(), table.numel(), None, int(length),
             query.shape[3] ** -0.5, _Pointers(query.data_ptr(), output.data_ptr()),
             (0, output.stride(1)))
        return output


def decode_attention_gqa(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor) -> torch.Tensor:
    """Online decode for Q [1,Hq,1,D] and original K/V [1,Hkv,L,D] (cuda_attention.py:63-83).

    Consecutive groups of Hq/Hkv query heads share each KV head; all L
    positions are attended; feature stride 1 and any nonnegative outer
    strides (cache-prefix views, zero-stride broadcasts) are read in place.
    float32/float16 in, fp32 accumulation, fresh contiguous output of Q's
    shape and dtype. Runs libmvdecode.so's contiguous-cache decode.
    """
    return _load_extension().decode_attention_gqa(query, key, value)


@lru_cache(maxsize=1)
def _load_extension() -> _DecodeAttentionExtension:
    _native.library()
    return _DecodeAttentionExtension()


def _is_paged_cache(cache) -> bool:
    """micro-vllm's ``PagedKVCache`` (src/micro_vllm/paged_kv_cache.py:43-199).

    Checked by class name and the attributes read here, so this package needs
    no import of micro-vllm: the reference's call site has already checked
    ``isinstance(cache, PagedKVCache)`` before calling (model.py:175-177).
    """
    return type(cache).__name__ == 'PagedKVCache' and all(
        hasattr(cache, name) for name in ('_keys', '_values', '_device_page_table', 'length',
                                          'num_kv_heads', 'head_dim', 'dtype', 'device'))


def _checked_paged_query(query, cache, layer_idx):
    if not _is_paged_cache(cache):
        raise ValueError('paged decode requires an owned PagedKVCache')
    length = cache.length(layer_idx)
    if length <= 0:
        raise ValueError('paged decode requires a nonempty cache layer')
    if not isinstance(query, torch.Tensor):
        raise ValueError('query must be a tensor')
    if query.layout != torch.strided or query.is_nested:
        raise ValueError('query must use dense strided storage')
    if (query.ndim != 4 or query.shape[0] != 1 or query.shape[1] <= 0
            or query.shape[2] != 1 or query.shape[3] != cache.head_dim):
        raise ValueError('query shape must be [1, query_heads, 1, cache.head_dim]')
    if query.shape[1] % cache.num_kv_heads:
        raise ValueError('query head count must be divisible by KV head count')
    if cache.dtype not in (torch.float16, torch.float32) or query.dtype != cache.dtype:
        raise ValueError('query and cache require matching float16 or float32 dtype')
    if query.requires_grad:
        raise ValueError('paged decode does not support gradients')
    if query.is_neg():
        raise ValueError('paged decode does not support lazy negative views')
    if query.stride(-1) != 1 or any(stride < 0 for stride in query.stride()[:-1]):
        raise ValueError('query requires feature stride 1 and nonnegative outer strides')
    if cache.device.type != 'cuda' or query.device != cache.device:
        raise ValueError('paged decode requires a CUDA cache and query on the same device')
    return length


@torch.inference_mode()
def decode_attention_paged(query: torch.Tensor, cache, *, layer_idx: int) -> torch.Tensor:
    """Attend the latest query directly over one owned PagedKVCache layer.

    Q is [1,Hq,1,D]; Hq is divisible by the cache's KV head count; every
    cached token including the current one is visible; fp16/fp32 I/O with fp32
    accumulation. No gather, KV repetition, host table read-back or
    context-sized score buffer. Output is fresh contiguous storage with the
    query's shape, device and dtype; inputs are unchanged.
    """
    length = _checked_paged_query(query, cache, layer_idx)
    return _load_extension()._decode_attention_paged(
        query, cache._keys[layer_idx], cache._values[layer_idx],
        cache._device_page_table, length)


# schedule keyword -> flag: the library's choice, the per-warp stream schedule
# wherever its shape allows, or never the stream schedule.
_SCHEDULES = {'auto': 0, 'stream': _native.FLAG_STREAM, 'split': _native.FLAG_SPLIT_GRID}


def _flags(force_simt, persistent, fused_merge=False, cluster=False, wide=False, cuda_core_math=False,
           schedule='auto'):
    _check(schedule in _SCHEDULES, "schedule must be 'auto', 'stream' or 'split'")
    return ((_native.FLAG_FORCE_SIMT if force_simt else 0) | (_native.FLAG_PERSISTENT if persistent else 0)
            | (_native.FLAG_FUSED_MERGE if fused_merge else 0) | (_native.FLAG_CLUSTER if cluster else 0)
            | (_native.FLAG_WIDE if wide else 0) | (_native.FLAG_CUDA_CORE_MATH if cuda_core_math else 0)
            | _SCHEDULES[schedule])


def _schedule_of(flags):
    for name, bit in _SCHEDULES.items():
        if bit and flags & bit:
            return name
    return 'auto'


# Plans whose tensor-core kernel rotates q and the new K rows itself (fused RoPE).
_ROPE_FUSED_TMA_PATHS = ('tma_mma', 'tma_mma_stream')


def paged_decode_plan(query_heads, key_cache, context_bound, *, batch, pages_per_split=0,
                      force_simt=False, persistent=False, cluster=False, wide=False, cuda_core_math=False,
                      schedule='auto'):
    """(path, pages_per_split, max_splits) that ``paged_decode_attention`` would use.

    path is 'tma_mma_stream' (TMA + tensor cores, one CTA per SM whose warps
    each stream pages of work items -- runs of pages_per_split pages of one
    sequence and KV head -- taken from a queue, merge pass), 'tma_mma_cluster'
    (TMA + tensor cores, the splits of each sequence/head in one thread-block
    cluster, combined through distributed shared memory), 'tma_mma' (TMA +
    tensor cores, one CTA per split of pages, merge pass), 'tma_mma_persistent'
    (TMA + tensor cores, a resident grid with equal page ranges per warp, merge
    pass) or 'simt' (CUDA cores, one CTA per split, merge pass).
    """
    lib = _native.library()
    num_blocks, kv_heads, block_size, dim = key_cache.shape
    path, pps, splits = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    with torch.cuda.device(key_cache.device):
        _native.check(lib.mv_paged_decode_plan(
            batch, query_heads, kv_heads, dim, block_size, context_bound, pages_per_split,
            _flags(force_simt, persistent, cluster=cluster, wide=wide, cuda_core_math=cuda_core_math,
                   schedule=schedule),
            DTYPE_CODES[key_cache.dtype],
            key_cache.data_ptr(), key_cache.data_ptr(), ctypes.byref(path), ctypes.byref(pps),
            ctypes.byref(splits)))
    return _native.PATH_NAMES[path.value], pps.value, splits.value


def paged_decode_attention(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                           block_table: torch.Tensor, context_lens: torch.Tensor,
                           scale: float | None = None, *, max_context_len: int | None = None,
                           out: torch.Tensor | None = None, pages_per_split: int = 0,
                           force_simt: bool = False, persistent: bool = False,
                           fused_merge: bool = False, cluster: bool = False, wide: bool = False,
                           cuda_core_math: bool = False, schedule: str = 'auto') -> torch.Tensor:
    """Batched paged GQA decode over one shared page pool.

    query: [B, Hq, D] (or [B, Hq, 1, D]) CUDA fp32/fp16/bf16, feature stride 1.
    key_cache/value_cache: [P, Hkv, bs, D] contiguous, same dtype.
    block_table: [B, max_blocks] int32/int64, contiguous rows.
    context_lens: [B] int32/int64 device tensor; tokens attended per sequence,
    including this step's appended token.
    scale: softmax scale (default head_dim ** -0.5, the reference's).
    max_context_len: host-side upper bound on context_lens; defaults to the
    table capacity max_blocks * bs, so no device read-back is needed. Lengths
    above it produce NaN (the split plan cannot cover them).
    out: optional [B, Hq, D] destination (feature stride 1).
    pages_per_split / cluster / persistent / fused_merge / wide / force_simt:
    kernel selection for tests and tuning (that many pages per split-KV CTA;
    the cluster kernel; the persistent tensor-core schedule; merging splits in
    the last split CTA; the split grid's wide shape of 8 warps with deeper
    rings; the CUDA-core kernel). cuda_core_math: the split grid's TMA pipeline
    with fp32 FMA math instead of the tensor-core tile (GQA group <= 8,
    head_dim 64/128; a comparison point). schedule: 'auto' (the library's
    choice), 'stream' (the per-warp stream schedule -- one CTA per SM, each
    warp streaming pages of work items from a queue; measured slower than the
    split grid, kept for comparison -- wherever its shape allows, else an
    error) or 'split' (the same as 'auto'). By default the library picks the
    tensor-core split grid with a merge pass, and the CUDA-core kernel for
    shapes the tensor-core kernels do not take.
    Returns out, or a fresh [B, Hq, D] tensor of the query's dtype.
    """
    q, max_context_len, scale, out = _checked_batched(query, key_cache, value_cache, block_table,
                                                      context_lens, scale, max_context_len, out)
    _launch_batched(q, key_cache, value_cache, block_table, context_lens, max_context_len, scale, out,
                    pages_per_split, _flags(force_simt, persistent, fused_merge, cluster, wide, cuda_core_math,
                                            schedule))
    return out


def _checked_batched(query, key_cache, value_cache, block_table, context_lens, scale, max_context_len,
                     out):
    """Validate the batched decode arguments; returns (q [B,Hq,D], bound, scale, out)."""
    squeeze = query.dim() == 4
    q = query[:, :, 0, :] if squeeze else query
    _check(isinstance(q, torch.Tensor) and q.dim() == 3, 'query must be [B, Hq, D] or [B, Hq, 1, D]')
    if squeeze:
        _check(query.shape[2] == 1, 'paged decode requires exactly one query token')
    for tensor in (q, key_cache, value_cache, block_table, context_lens):
        _validate_storage(tensor)
    _check(q.dtype in DTYPE_CODES, 'query must be float32, float16 or bfloat16')
    _check(q.dtype == key_cache.dtype == value_cache.dtype, 'Q and K/V pages must use the same dtype')
    _check(q.device == key_cache.device == value_cache.device == block_table.device
           == context_lens.device, 'Q, K/V pages, table and lengths must use the same device')
    _check(key_cache.dim() == 4 and key_cache.shape == value_cache.shape,
           'K/V pages must both have shape [P,Hkv,B,D]')
    _check(key_cache.is_contiguous() and value_cache.is_contiguous(), 'K/V pages must be contiguous')
    batch, q_heads, dim = q.shape
    num_blocks, kv_heads, block_size, kdim = key_cache.shape
    _check(batch > 0 and q_heads > 0 and dim > 0 and key_cache.numel() > 0,
           'page dimensions, head counts, and head dimension must be positive')
    _check(dim == kdim, 'Q and K/V pages must share the head dimension')
    _check(q_heads % kv_heads == 0, 'query head count must be divisible by KV head count')
    _check(q.stride(2) == 1 and q.stride(0) >= 0 and q.stride(1) >= 0,
           'query requires feature stride 1 and nonnegative outer strides')
    _check(block_table.dtype in INDEX_CODES and context_lens.dtype in INDEX_CODES,
           'block table and context lengths must be int32 or int64')
    _check(block_table.dim() == 2 and block_table.shape[0] == batch and block_table.shape[1] > 0,
           'block table must have shape [B, max_blocks]')
    _check(block_table.stride(1) == 1 and (batch == 1 or block_table.stride(0) >= block_table.shape[1]),
           'block table rows must be contiguous')
    _check(context_lens.shape == (batch,) and context_lens.is_contiguous(),
           'context lengths must be a contiguous [B] tensor')
    capacity = block_table.shape[1] * block_size
    if max_context_len is None:
        max_context_len = capacity
    _check(0 <= max_context_len, 'max_context_len must be nonnegative')
    if scale is None:
        scale = dim ** -0.5
    if out is None:
        out = torch.empty((batch, q_heads, dim), dtype=q.dtype, device=q.device)
    else:
        _validate_storage(out)
        _check(out.shape == (batch, q_heads, dim) and out.dtype == q.dtype and out.device == q.device,
               'out must be a [B, Hq, D] tensor of the query dtype and device')
        _check(out.stride(2) == 1, 'out requires feature stride 1')
    return q, max_context_len, scale, out


def _launch_batched(q, key_cache, value_cache, block_table, context_lens, max_context_len, scale, out,
                    pages_per_split, flags, rows=None):
    batch, q_heads, dim = q.shape
    _run((batch, q_heads, dim), (q.stride(0), q.stride(1)), key_cache, value_cache, block_table,
         block_table.stride(0), block_table.shape[1], context_lens, int(max_context_len), scale,
         _Pointers(q.data_ptr(), out.data_ptr()), (out.stride(0), out.stride(1)),
         pages_per_split=int(pages_per_split), flags=flags, rows=rows)


def paged_decode_with_append(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                             key_cache: torch.Tensor, value_cache: torch.Tensor,
                             block_table: torch.Tensor, context_lens: torch.Tensor,
                             scale: float | None = None, *, max_context_len: int | None = None,
                             out: torch.Tensor | None = None, pages_per_split: int = 0,
                             force_simt: bool = False, persistent: bool = False,
                             fused_merge: bool = False, cluster: bool = False, wide: bool = False,
                             rope: tuple[torch.Tensor, torch.Tensor] | None = None,
                             cuda_core_math: bool = False, schedule: str = 'auto') -> torch.Tensor:
    """One decode step of a layer: append this step's K/V row of every sequence, then attend.

    The result, in the pools and in the output, is that of
    ``write_paged_kv(key, value, key_cache, value_cache, block_table,
    positions=context_lens, positions_are_end=True)`` followed by
    ``paged_decode_attention(query, key_cache, value_cache, block_table,
    context_lens, scale)`` -- the append-before-attend order of the
    reference's decode layer (src/micro_vllm/model.py:215-216) -- but where
    the stream schedule, the split-grid tensor-core kernel or the CUDA-core
    kernel runs, the warp or CTA attending each sequence's last page writes the
    new row itself, so the step is one kernel (plus the split merge) instead
    of two. The persistent and cluster schedules run the append kernel first.

    key/value: [B, Hkv, D] or [B, Hkv, 1, D] CUDA tensors of the pool dtype,
    feature stride 1. context_lens count the new token. The page receiving a
    sequence's new row must not be shared with another sequence of the batch.
    rope: optional (cos, sin) tables ``rope.rope_tables`` builds; q and key are
    then unrotated and get RoPE at position context_lens - 1 (the reference's
    apply_rope before the append, model.py:214-215) -- inside the decode kernel
    on the fused path, else by the RoPE kernel first.
    Other arguments as ``paged_decode_attention``. Returns out.
    """
    from . import cuda_paged_cache as cache_ops

    q, max_context_len, scale, out = _checked_batched(query, key_cache, value_cache, block_table,
                                                      context_lens, scale, max_context_len, out)
    key4 = key.unsqueeze(2) if key.dim() == 3 else key
    value4 = value.unsqueeze(2) if value.dim() == 3 else value
    for tensor in (key4, value4):
        cache_ops._validate_data(tensor, key_cache)
    cache_ops._validate_sources(key4, value4, batched=True)
    _check(key4.shape[0] == q.shape[0] and key4.shape[2] == 1,
           'new K/V must have shape [B, Hkv, D] or [B, Hkv, 1, D]')
    cache_ops._validate_pages(key4, key_cache, value_cache)
    cache_ops._validate_aliases(key4, value4, key_cache, value_cache, block_table)
    flags = _flags(force_simt, persistent, fused_merge, cluster, wide, cuda_core_math, schedule)
    key3, value3 = key4[:, :, 0, :], value4[:, :, 0, :]
    tables = None
    if rope is not None:
        from . import rope as rope_ops
        cos, sin = rope
        rope_ops.check_tables(cos, sin, q.shape[2], q.dtype, q.device)
        path = paged_decode_plan(q.shape[1], key_cache, max_context_len, batch=q.shape[0],
                                 pages_per_split=pages_per_split, force_simt=force_simt,
                                 persistent=persistent, cluster=cluster, wide=wide,
                                 cuda_core_math=cuda_core_math, schedule=schedule)[0]
        if (path in _ROPE_FUSED_TMA_PATHS and _aligned16(key3, value3, cos, sin)) or path == 'simt':
            tables = (cos, sin)
        else:
            q = rope_ops.apply_rope(q, cos, sin, positions=context_lens, positions_are_end=True)
            key3 = rope_ops.apply_rope(key3, cos, sin, positions=context_lens, positions_are_end=True)
    _launch_batched(q, key_cache, value_cache, block_table, context_lens, max_context_len, scale, out,
                    pages_per_split, flags, rows=(key3, value3, tables))
    return out


def _aligned16(*tensors):
    """Every tensor's start and outer element strides are 16-byte multiples (2-byte types)."""
    for t in tensors:
        if t.data_ptr() % 16 or any((t.stride(d) * t.element_size()) % 16 for d in range(t.dim() - 1)):
            return False
    return True


def _data_ptrs(*tensors):
    """Storage addresses and strides: a repeat must see the same views, not only the same memory."""
    return tuple((t.data_ptr(), t.stride()) if t is not None else (0, ()) for t in tensors)


class PagedDecodeStep:
    """A decode step bound to one page pool, validated once and called per step.

    The serving loop calls the same layer geometry every step: the pools, the
    block table tensor, the head counts, the context bound, the scale and the
    kernel choice do not change, only the query, this step's new K/V rows, the
    lengths (device data) and the output. Binding them once moves every check
    that ``paged_decode_attention`` / ``paged_decode_with_append`` repeat per
    call to construction, so a call costs a few attribute comparisons and one
    C-ABI call (``mv_paged_decode_step_args``: the arguments of
    ``mv_paged_decode`` / ``mv_paged_decode_append`` in one struct, filled at
    construction and on each validated call). A call repeating one of the
    last eight validated ones -- the same tensor objects over the same
    storage with the same strides, on the same stream, with a caller-given
    output -- skips even
    those comparisons; the step keeps references to those tensors until they
    are evicted. Results are identical to those functions on the same
    arguments.

    ``step(query, context_lens, out=None, key=None, value=None)``: query
    [B, Hq, D] or [B, Hq, 1, D]; context_lens [B] int32/int64 on the pool's
    device; key/value (both or neither) [B, Hkv, D] or [B, Hkv, 1, D], appended
    at position context_lens - 1 before attending. With ``rope=(cos, sin)``
    bound, q and key arrive unrotated and are rotated at that position (inside
    the decode kernel where it can, else by the RoPE kernel first). The block
    table's contents may change between calls; its tensor (pointer, shape) may
    not. Calls on one stream share one split-KV workspace and must be ordered on it.
    """

    def __init__(self, key_cache: torch.Tensor, value_cache: torch.Tensor, block_table: torch.Tensor, *,
                 num_q_heads: int, max_context_len: int | None = None, scale: float | None = None,
                 pages_per_split: int = 0, force_simt: bool = False, persistent: bool = False,
                 fused_merge: bool = False, cluster: bool = False, wide: bool = False,
                 rope: tuple[torch.Tensor, torch.Tensor] | None = None, schedule: str = 'auto'):
        batch = block_table.shape[0] if block_table.dim() == 2 else 0
        dim = key_cache.shape[-1] if key_cache.dim() == 4 else 0
        probe = torch.empty((max(batch, 1), num_q_heads, max(dim, 1)), dtype=key_cache.dtype,
                            device=key_cache.device)
        lens = torch.empty((max(batch, 1),), dtype=torch.int32, device=key_cache.device)
        _, bound, scale, _ = _checked_batched(probe, key_cache, value_cache, block_table, lens, scale,
                                              max_context_len, probe)
        self._lib = _native.library()
        self._device = key_cache.device
        self._device_index = key_cache.device.index
        self._dtype = key_cache.dtype
        num_blocks, kv_heads, block_size, _ = key_cache.shape
        self._q_shape = (batch, num_q_heads, dim)
        self._row_shape = (batch, kv_heads, dim)
        self._flags = _flags(force_simt, persistent, fused_merge, cluster, wide, schedule=schedule)
        self._pps = int(pages_per_split)
        self._bound = int(bound)
        self._pools = (key_cache, value_cache)
        self._table = block_table
        nbytes = key_cache.numel() * key_cache.element_size()
        self._pool_ranges = ((key_cache.data_ptr(), key_cache.data_ptr() + nbytes),
                             (value_cache.data_ptr(), value_cache.data_ptr() + nbytes))
        dtype = DTYPE_CODES[key_cache.dtype]
        size = ctypes.c_size_t(0)
        with torch.cuda.device(self._device):
            _native.check(self._lib.mv_paged_decode_workspace_size(
                batch, num_q_heads, kv_heads, dim, block_size, self._bound, self._pps, self._flags, dtype,
                ctypes.byref(size)))
        self._workspace_bytes = size.value
        self._scale = float(scale)
        self._dtype_code = dtype
        # The call's arguments in one struct (mv_paged_decode_step_args): the
        # bound fields are set once, the per-call ones on each validated call.
        self._args = _native.MvDecodeStepArgs(
            k_cache=key_cache.data_ptr(), v_cache=value_cache.data_ptr(), num_blocks=num_blocks,
            num_kv_heads=kv_heads, block_size=block_size, head_dim=dim, block_table=block_table.data_ptr(),
            block_table_type=INDEX_CODES[block_table.dtype], block_table_stride=block_table.stride(0),
            blocks_per_seq=block_table.shape[1], max_context_len=self._bound, batch=batch,
            num_q_heads=num_q_heads, scale=self._scale, workspace_bytes=self._workspace_bytes,
            pages_per_split=self._pps, flags=self._flags, dtype=dtype)
        self._args_ref = ctypes.byref(self._args)
        # Validated calls a repeat may skip the checks for (a serving loop
        # cycles through a few static buffer sets): object ids -> (the
        # objects, their data pointers, stream, workspace, packed arguments).
        # Holding the objects keeps them, and so their ids, alive.
        self._fast = {}
        self._rope = None
        self._rope_in_kernel = False
        if rope is not None:
            from . import rope as rope_ops
            rope_ops.check_tables(rope[0], rope[1], dim, key_cache.dtype, key_cache.device)
            self._rope = (rope[0], rope[1])
            path = self.plan[0]
            self._rope_kernel_path = path
            self._rope_in_kernel = (path in _ROPE_FUSED_TMA_PATHS and _aligned16(*rope)) or path == 'simt'

    @property
    def plan(self):
        """(path, pages_per_split, max_splits) of the bound geometry."""
        return paged_decode_plan(self._q_shape[1], self._pools[0], self._bound, batch=self._q_shape[0],
                                 pages_per_split=self._pps,
                                 force_simt=bool(self._flags & _native.FLAG_FORCE_SIMT),
                                 persistent=bool(self._flags & _native.FLAG_PERSISTENT),
                                 cluster=bool(self._flags & _native.FLAG_CLUSTER),
                                 wide=bool(self._flags & _native.FLAG_WIDE),
                                 schedule=_schedule_of(self._flags))

    def _check_rows(self, rows):
        if rows.dim() == 4:
            _check(rows.shape[2] == 1, 'new K/V must have shape [B, Hkv, D] or [B, Hkv, 1, D]')
            rows = rows[:, :, 0]
        _check(tuple(rows.shape) == self._row_shape and rows.dtype == self._dtype
               and rows.device == self._device, 'new K/V must be [B, Hkv, D] rows of the pool dtype and device')
        _check(rows.stride(2) == 1 and rows.stride(0) >= 0 and rows.stride(1) >= 0 and not rows.requires_grad,
               'K/V require feature stride 1 and nonnegative outer strides')
        start = rows.data_ptr()
        for lo, hi in self._pool_ranges:
            _check(not (lo <= start < hi), 'sources and page table must not alias destination storage')
        return rows

    def __call__(self, query: torch.Tensor, context_lens: torch.Tensor, out: torch.Tensor | None = None,
                 key: torch.Tensor | None = None, value: torch.Tensor | None = None) -> torch.Tensor:
        # A repeat of the last call -- the same tensor objects over the same
        # storage, on the same stream (a serving loop's static buffers) -- was
        # validated then: only the C call remains (a few us of host time
        # instead of ~45 for the checks and a 35-argument ctypes call).
        ids = (id(query), id(context_lens), id(out), id(key), id(value))
        entry = self._fast.get(ids)
        if entry is not None and torch.cuda.current_device() == self._device_index:
            objects, ptrs, stream0, _, args_ref = entry
            stream = current_stream_raw(self._device_index)
            if (stream == stream0 and objects[0] is query and objects[2] is out
                    and ptrs == _data_ptrs(query, context_lens, out, key, value)):
                _native.check(self._lib.mv_paged_decode_step_args(args_ref, stream))
                return out
        self._fast.pop(ids, None)
        out_given = out is not None
        q = query[:, :, 0] if query.dim() == 4 and query.shape[2] == 1 else query
        _check(tuple(q.shape) == self._q_shape and q.dtype == self._dtype and q.device == self._device,
               'query must be [B, Hq, D] (or [B, Hq, 1, D]) of the bound shape, dtype and device')
        _check(q.stride(2) == 1 and q.stride(0) >= 0 and q.stride(1) >= 0 and not q.requires_grad,
               'query requires feature stride 1 and nonnegative outer strides')
        lens_code = INDEX_CODES.get(context_lens.dtype)
        _check(lens_code is not None and tuple(context_lens.shape) == self._q_shape[:1]
               and context_lens.device == self._device and context_lens.is_contiguous(),
               'context lengths must be a contiguous [B] int32/int64 tensor on the pool device')
        if out is None:
            out = torch.empty(self._q_shape, dtype=self._dtype, device=self._device)
        else:
            _check(tuple(out.shape) == self._q_shape and out.dtype == self._dtype and out.device == self._device
                   and out.stride(2) == 1, 'out must be a [B, Hq, D] tensor of the query dtype and device')
        _check((key is None) == (value is None), 'pass both new K and V rows, or neither')
        if torch.cuda.current_device() != self._device_index:
            with torch.cuda.device(self._device):
                return self(query, context_lens, out if out_given else None, key, value)
        stream = current_stream_raw(self._device_index)
        workspace = _workspace(self._device, stream, self._workspace_bytes) if self._workspace_bytes else None
        a = self._args
        a.q, a.q_stride_seq, a.q_stride_head = q.data_ptr(), q.stride(0), q.stride(1)
        a.context_lens, a.context_lens_type = context_lens.data_ptr(), lens_code
        a.out, a.out_stride_seq, a.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
        a.workspace = workspace.data_ptr() if workspace is not None else None
        rotated_here = False
        if key is None:
            _check(self._rope is None, 'a step bound with RoPE tables needs the new K/V rows')
            a.key = a.value = a.rope_cos = a.rope_sin = None
            a.key_stride_seq = a.key_stride_head = a.value_stride_seq = a.value_stride_head = a.rope_rows = 0
        else:
            rows_k, rows_v = self._check_rows(key), self._check_rows(value)
            a.rope_cos = a.rope_sin = None
            a.rope_rows = 0
            if self._rope is not None:
                cos, sin = self._rope
                if self._rope_in_kernel and (self._rope_kernel_path == 'simt' or _aligned16(rows_k, rows_v)):
                    a.rope_cos, a.rope_sin, a.rope_rows = cos.data_ptr(), sin.data_ptr(), cos.shape[0]
                else:
                    from . import rope as rope_ops
                    q = rope_ops.apply_rope(q, cos, sin, positions=context_lens, positions_are_end=True)
                    rows_k = rope_ops.apply_rope(rows_k, cos, sin, positions=context_lens, positions_are_end=True)
                    a.q, a.q_stride_seq, a.q_stride_head = q.data_ptr(), q.stride(0), q.stride(1)
                    rotated_here = True
            a.key, a.key_stride_seq, a.key_stride_head = rows_k.data_ptr(), rows_k.stride(0), rows_k.stride(1)
            a.value, a.value_stride_seq, a.value_stride_head = rows_v.data_ptr(), rows_v.stride(0), rows_v.stride(1)
        _native.check(self._lib.mv_paged_decode_step_args(self._args_ref, stream))
        if out_given and not rotated_here and not torch.cuda.is_current_stream_capturing():
            if len(self._fast) >= 8:
                self._fast.pop(next(iter(self._fast)))
            args = _native.MvDecodeStepArgs()
            ctypes.pointer(args)[0] = a
            self._fast[ids] = ((query, context_lens, out, key, value),
                               _data_ptrs(query, context_lens, out, key, value), stream, workspace,
                               ctypes.byref(args))
        return out


def contiguous_decode_attention(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                                context_lens: torch.Tensor | None = None, scale: float | None = None, *,
                                max_context_len: int | None = None, out: torch.Tensor | None = None,
                                pages_per_split: int = 0, force_simt: bool = False,
                                wide: bool = False) -> torch.Tensor:
    """Batched GQA decode over contiguous caches (the batched form of ``decode_attention_gqa``).

    query: [B, Hq, D] or [B, Hq, 1, D]; key_cache/value_cache: [B, Hkv, L, D]
    views with feature stride 1 and any nonnegative outer strides (e.g. the
    prefix of a larger cache buffer); context_lens: optional [B] int32/int64
    device lengths (<= L), else every sequence attends max_context_len
    (default L) tokens. fp32/fp16/bf16. Returns out ([B, Hq, D]).
    """
    squeeze = query.dim() == 4
    q = query[:, :, 0, :] if squeeze else query
    _check(isinstance(q, torch.Tensor) and q.dim() == 3, 'query must be [B, Hq, D] or [B, Hq, 1, D]')
    for tensor in (q, key_cache, value_cache) + ((context_lens,) if context_lens is not None else ()):
        _validate_storage(tensor)
    _check(q.dtype in DTYPE_CODES and q.dtype == key_cache.dtype == value_cache.dtype,
           'Q and K/V caches must share a float32, float16 or bfloat16 dtype')
    _check(q.device == key_cache.device == value_cache.device, 'Q and K/V caches must use the same device')
    _check(key_cache.dim() == 4 and key_cache.shape == value_cache.shape,
           'K/V caches must both have shape [B,Hkv,L,D]')
    batch, q_heads, dim = q.shape
    _check(key_cache.shape[0] == batch and key_cache.shape[3] == dim and batch > 0 and q_heads > 0
           and key_cache.numel() > 0, 'K/V caches must match the query batch and head dimension')
    _check(q_heads % key_cache.shape[1] == 0, 'query head count must be divisible by KV head count')
    for tensor in (q, key_cache, value_cache):
        _check(tensor.stride(-1) == 1 and all(tensor.stride(d) >= 0 for d in range(tensor.dim() - 1)),
               'tensors require feature stride 1 and nonnegative outer strides')
    if context_lens is not None:
        _check(context_lens.dtype in INDEX_CODES and context_lens.shape == (batch,)
               and context_lens.is_contiguous() and context_lens.device == q.device,
               'context lengths must be a contiguous [B] int32/int64 tensor on the query device')
    cache_len = key_cache.shape[2]
    bound = cache_len if max_context_len is None else int(max_context_len)
    _check(bound >= 0, 'max_context_len must be nonnegative')
    if scale is None:
        scale = dim ** -0.5
    if out is None:
        out = torch.empty((batch, q_heads, dim), dtype=q.dtype, device=q.device)
    else:
        _validate_storage(out)
        _check(out.shape == (batch, q_heads, dim) and out.dtype == q.dtype and out.device == q.device
               and out.stride(2) == 1, 'out must be a [B, Hq, D] tensor of the query dtype and device')
    _run_contiguous((batch, q_heads, dim), (q.stride(0), q.stride(1)), key_cache, value_cache, context_lens,
                    bound, scale, _Pointers(q.data_ptr(), out.data_ptr()), (out.stride(0), out.stride(1)),
                    pages_per_split=int(pages_per_split), flags=_flags(force_simt, False, wide=wide))
    return out


def contiguous_decode_plan(key_cache, value_cache, query_heads, *, max_context_len=None, pages_per_split=0,
                           force_simt=False, wide=False):
    """(path, pages_per_split, max_splits) that ``contiguous_decode_attention`` would use."""
    lib = _native.library()
    batch, kv_heads, cache_len, dim = key_cache.shape
    bound = cache_len if max_context_len is None else int(max_context_len)
    path, pps, splits = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    size = ctypes.c_size_t(0)
    with torch.cuda.device(key_cache.device):
        _native.check(lib.mv_contiguous_decode_plan(
            key_cache.data_ptr(), key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
            value_cache.data_ptr(), value_cache.stride(0), value_cache.stride(1), value_cache.stride(2),
            cache_len, kv_heads, dim, bound, batch, query_heads, pages_per_split,
            _flags(force_simt, False, wide=wide), DTYPE_CODES[key_cache.dtype], ctypes.byref(path),
            ctypes.byref(pps), ctypes.byref(splits), ctypes.byref(size)))
    return _native.PATH_NAMES[path.value], pps.value, splits.value


def paged_chunk_attention(query: torch.Tensor, key_cache: torch.Tensor, value_cache: torch.Tensor,
                          block_table: torch.Tensor, context_lens: torch.Tensor, scale: float | None = None, *,
                          max_context_len: int | None = None, out: torch.Tensor | None = None,
                          pages_per_split: int = 0, force_simt: bool = False,
                          kernel: str = 'auto') -> torch.Tensor:
    """Causal attention of a chunk of T new tokens per sequence over its pages.

    query: [B, Hq, T, D] (the reference's layout for a cached chunk), feature
    stride 1. The chunk's K/V must already be appended; context_lens [B]
    counts each sequence's tokens after the chunk, and token t attends the
    first context_lens - (T - 1 - t) of them (model.py:178-182 gathers the
    pages and runs causal attention for this; nothing is gathered here).
    ``kernel``: 'auto' runs query tiles on tensor cores where the shape allows
    (fp16/bf16, head_dim 64/128, 16-token pages, T x G >= 16 rows per KV
    head): 128 rows per CTA on tcgen05 from 64 rows up with a 16-byte aligned
    query, else 64 rows per CTA on mma.sync; 'mma_sync' forces the 64-row
    tiles; 'rows' (or an ineligible shape) runs one decode query row per token.
    Other arguments as ``paged_decode_attention``. Returns [B, Hq, T, D].
    """
    _check(isinstance(query, torch.Tensor) and query.dim() == 4, 'query must be [B, Hq, T, D]')
    batch, q_heads, tokens, dim = query.shape
    # Validate with one token's view; the token stride is passed separately.
    q0, bound, scale, _ = _checked_batched(query[:, :, 0, :], key_cache, value_cache, block_table, context_lens,
                                           scale, max_context_len, None)
    _check(tokens > 0 and query.stride(2) >= 0, 'query requires a positive token count and nonnegative strides')
    if out is None:
        out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    else:
        _validate_storage(out)
        _check(out.shape == query.shape and out.dtype == query.dtype and out.device == query.device
               and out.stride(3) == 1, 'out must be a [B, Hq, T, D] tensor of the query dtype and device')
    lib = _native.library()
    num_blocks, kv_heads, block_size, _ = key_cache.shape
    _check(kernel in ('auto', 'mma_sync', 'rows'), "kernel must be 'auto', 'mma_sync' or 'rows'")
    flags = _flags(force_simt, False) | {'auto': 0, 'mma_sync': _native.FLAG_CHUNK_MMA_SYNC,
                                         'rows': _native.FLAG_CHUNK_ROWS}[kernel]
    dtype = DTYPE_CODES[key_cache.dtype]
    device = key_cache.device
    with torch.cuda.device(device):
        size = ctypes.c_size_t(0)
        _native.check(lib.mv_paged_chunk_workspace_size(
            batch, tokens, q_heads, kv_heads, dim, block_size, int(bound), int(pages_per_split), flags, dtype,
            ctypes.byref(size)))
        stream = current_stream_handle(device)
        workspace = _workspace(device, stream, size.value) if size.value else None
        _native.check(lib.mv_paged_chunk_attention(
            query.data_ptr(), query.stride(0), query.stride(2), query.stride(1),
            key_cache.data_ptr(), value_cache.data_ptr(), num_blocks, kv_heads, block_size, dim,
            block_table.data_ptr(), INDEX_CODES[block_table.dtype], block_table.stride(0), block_table.shape[1],
            context_lens.data_ptr(), INDEX_CODES[context_lens.dtype], int(bound), batch, tokens, q_heads,
            float(scale), out.data_ptr(), out.stride(0), out.stride(2), out.stride(1),
            workspace.data_ptr() if workspace is not None else None,
            workspace.numel() if workspace is not None else 0, int(pages_per_split), flags, dtype, stream))
    return out
