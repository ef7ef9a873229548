"""Native paged K/V writes: drop-in for ``micro_vllm.cuda_paged_cache``.

``_write_paged_kv`` keeps the reference's signature, argument meaning and
error messages (src/micro_vllm/cuda_paged_cache.py:23-41 and the checks of
src/micro_vllm/csrc/paged_kv_cache.cpp:19-107), but runs the sm_100a
vectorised scatter kernel of libmvdecode.so through its C ABI
(``mv_write_paged_kv``). ``write_paged_kv`` is the batched form: one launch
appends N tokens for each of B sequences through their block-table rows.

Importing this module loads nothing; the library is opened on first use.
There is no CPU path: non-CUDA tensors are rejected.
"""
from functools import lru_cache

import torch

from . import _native
from ._tensors import DTYPE_CODES, INDEX_CODES, current_stream_handle, storage_overlaps

_INT64_MAX = 2 ** 63 - 1


def _check(condition, message):
    if not condition:
        raise RuntimeError(message)


def _validate_storage(tensor):
    _check(tensor.is_cuda, 'paged KV writes require CUDA tensors')
    _check(tensor.layout == torch.strided and not tensor.is_nested,
           'paged KV writes require strided tensors')
    _check(not tensor.requires_grad, 'paged KV writes do not support gradients')
    _check(not tensor.is_neg(), 'paged KV writes do not support lazy negative views')


def _validate_data(tensor, key):
    _validate_storage(tensor)
    _check(tensor.dtype in DTYPE_CODES, 'paged KV writes require float16, bfloat16 or float32 dtype')
    _check(tensor.dtype == key.dtype, 'K/V and pages must have the same dtype')
    _check(tensor.device == key.device, 'all tensors must use the same device')


def _validate_sources(key, value, batched):
    _check(key.dim() == 4 and value.dim() == 4,
           'K/V must have shape [B,H,N,D]' if batched else 'K/V must have shape [1,H,N,D]')
    _check(key.shape == value.shape, 'K/V must have the same shape')
    if not batched:
        _check(key.shape[0] == 1, 'K/V shape requires batch size 1')
    _check(key.numel() > 0, 'K/V head, token and feature dimensions must be positive')
    for source in (key, value):
        _check(source.stride(3) == 1, 'K/V require feature stride 1')
        _check(all(source.stride(d) >= 0 for d in range(3)), 'K/V require nonnegative outer strides')


def _validate_pages(key, key_pages, value_pages):
    _check(key_pages.dim() == 4 and value_pages.dim() == 4, 'pages must have shape [P,H,B,D]')
    _check(key_pages.shape == value_pages.shape, 'K/V pages must have the same shape')
    _check(key_pages.numel() > 0, 'page dimensions must be positive')
    _check(key_pages.shape[1] == key.shape[1] and key_pages.shape[3] == key.shape[3],
           'page shape must match K/V head count and feature dimension')
    _check(key_pages.is_contiguous() and value_pages.is_contiguous(), 'K/V pages must be contiguous')


def _validate_table(table, pages, start, tokens):
    _validate_storage(table)
    _check(table.device == pages.device, 'all tensors must use the same device')
    _check(table.dtype == torch.int64, 'page table must use int64 dtype')
    _check(table.dim() == 1, 'page table must be one-dimensional (1D)')
    _check(table.numel() > 0, 'page table must be nonempty')
    _check(table.is_contiguous(), 'page table must be contiguous')
    _check(table.numel() <= pages.shape[0], 'page table cannot exceed physical page capacity')
    _check(table.numel() <= _INT64_MAX // pages.shape[2], 'page table capacity is too large')
    capacity = table.numel() * pages.shape[2]
    _check(0 <= start <= capacity, 'start must lie within cache capacity')
    _check(tokens <= capacity - start, 'append exceeds cache capacity')


def _validate_aliases(key, value, key_pages, value_pages, table):
    _check(not storage_overlaps(key_pages, value_pages), 'K/V pages must not alias storage')
    for source in (key, value, table):
        _check(not storage_overlaps(source, key_pages) and not storage_overlaps(source, value_pages),
               'sources and page table must not alias destination storage')


def _launch(key, value, key_pages, value_pages, table, table_stride, blocks_per_seq,
            positions, positions_kind, start):
    lib = _native.library()
    batch, heads, tokens, dim = key.shape
    device = key_pages.device
    with torch.cuda.device(device):
        _native.check(lib.mv_write_paged_kv(
            key.data_ptr(), key.stride(0), key.stride(1), key.stride(2),
            value.data_ptr(), value.stride(0), value.stride(1), value.stride(2),
            key_pages.data_ptr(), value_pages.data_ptr(), key_pages.shape[0],
            heads, key_pages.shape[2], dim,
            table.data_ptr(), INDEX_CODES[table.dtype], table_stride, blocks_per_seq,
            positions.data_ptr() if positions is not None else None,
            INDEX_CODES[positions.dtype] if positions is not None else 0,
            positions_kind, start, batch, tokens, DTYPE_CODES[key.dtype],
            current_stream_handle(device)))


class _PagedCacheExtension:
    """The object ``_load_extension()`` returns, shaped like the reference's pybind module."""

    def write_paged_kv(self, key, value, key_pages, value_pages, page_table, start):
        """Validate like paged_kv_cache.cpp:96-107, then launch the append kernel."""
        for tensor in (key, value, key_pages, value_pages):
            _validate_data(tensor, key)
        _validate_sources(key, value, batched=False)
        _validate_pages(key, key_pages, value_pages)
        if type(start) is not int:
            raise TypeError('start must be an int')
        _validate_table(page_table, key_pages, start, key.shape[2])
        _validate_aliases(key, value, key_pages, value_pages, page_table)
        _launch(key, value, key_pages, value_pages, page_table, 0, page_table.numel(),
                None, _native.POSITIONS_START, start)


@lru_cache(maxsize=1)
def _load_extension() -> _PagedCacheExtension:
    _native.library()
    return _PagedCacheExtension()


def _write_paged_kv(key: torch.Tensor, value: torch.Tensor,
                    key_pages: torch.Tensor, value_pages: torch.Tensor,
                    page_table: torch.Tensor, start: int) -> None:
    """Copy post-RoPE K/V [1,H,N,D] into fixed [P,H,B,D] pages at ``start``.

    Same contract as the reference helper: metadata is validated on the host
    with no GPU-to-host synchronisation; corrupted physical IDs in the device
    table are skipped by the kernel, never written out of bounds; copies are
    bit-exact for fp16/bf16/fp32; work runs on the current CUDA stream.
    """
    _load_extension().write_paged_kv(key, value, key_pages, value_pages, page_table, start)


def write_paged_kv(key: torch.Tensor, value: torch.Tensor,
                   key_cache: torch.Tensor, value_cache: torch.Tensor,
                   block_table: torch.Tensor, *, positions: torch.Tensor | None = None,
                   start: int = 0, positions_are_end: bool = False) -> None:
    """Batched append: token t of sequence b lands at logical position start_b + t.

    key/value: [B, Hkv, N, D] CUDA, feature stride 1 (any nonnegative outer
    strides). key_cache/value_cache: [P, Hkv, bs, D] contiguous.
    block_table: [B, max_blocks] int32/int64 with contiguous rows.
    positions: optional [B] int32/int64 device tensor giving start_b, or the
    sequence length after the append when ``positions_are_end`` (decode:
    pass the context lengths and the new token lands at length - 1);
    without it every sequence starts at ``start``. Positions are device data:
    tokens that fall outside the table row, or on an out-of-range physical
    page ID, are skipped rather than written out of bounds.
    """
    for tensor in (key, value, key_cache, value_cache):
        _validate_data(tensor, key)
    _validate_sources(key, value, batched=True)
    _validate_pages(key, key_cache, value_cache)
    _validate_storage(block_table)
    _check(block_table.device == key_cache.device, 'all tensors must use the same device')
    _check(block_table.dtype in INDEX_CODES, 'block table must use int32 or int64 dtype')
    _check(block_table.dim() == 2 and block_table.shape[0] == key.shape[0]
           and block_table.shape[1] > 0, 'block table must have shape [B, max_blocks]')
    _check(block_table.stride(1) == 1 and block_table.stride(0) >= block_table.shape[1],
           'block table rows must be contiguous')
    if positions is not None:
        _validate_storage(positions)
        _check(positions.device == key_cache.device, 'all tensors must use the same device')
        _check(positions.dtype in INDEX_CODES, 'positions must use int32 or int64 dtype')
        _check(positions.shape == (key.shape[0],) and positions.is_contiguous(),
               'positions must be a contiguous [B] tensor')
    _validate_aliases(key, value, key_cache, value_cache, block_table)
    kind = _native.POSITIONS_END if positions_are_end else _native.POSITIONS_START
    _launch(key, value, key_cache, value_cache, block_table, block_table.stride(0),
            block_table.shape[1], positions, kind, int(start))
