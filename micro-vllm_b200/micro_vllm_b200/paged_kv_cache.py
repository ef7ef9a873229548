"""Fixed-page KV storage for one request on a CUDA device.

Same layout, contract and messages as the reference's ``PagedKVCache``
(src/micro_vllm/paged_kv_cache.py:43-199): per layer, K and V pools of shape
[num_pages, kv_heads, page_size, head_dim]; an immutable host page table
validated once at allocation and a private int64 device copy of it; appends
validated before any write; ``reset`` hides tokens and keeps storage.

Differences, by design: storage must be on a CUDA device (appends always run
the native kernel; there is no CPU path), and the dataclass constructor may be
given externally owned pools, so several single-request caches can share one
pool (the batched decode harness does this).
"""
from collections.abc import Sequence
from dataclasses import dataclass, field

import torch

from ._tensors import storage_overlaps


def _checked_page_ids(page_table, num_pages):
    if page_table is None:
        return tuple(range(num_pages))
    if not isinstance(page_table, Sequence) or isinstance(page_table, (str, bytes)):
        raise ValueError('page_table must be a sequence of physical page IDs')
    page_ids = tuple(page_table)
    if (not page_ids or any(type(page) is not int or not 0 <= page < num_pages
                            for page in page_ids)):
        raise ValueError('page_table must contain nonempty integer IDs within the physical pool')
    if len(set(page_ids)) != len(page_ids):
        raise ValueError('page_table must not assign a physical page more than once')
    return page_ids


@dataclass
class PagedKVCache:
    """Fixed single-request mapping; append/reset mutate storage and return self."""

    _keys: tuple = field(repr=False)
    _values: tuple = field(repr=False)
    _lengths: list
    _page_ids: tuple
    _device_page_table: torch.Tensor = field(repr=False)

    @classmethod
    def allocate(cls, *, num_layers, num_kv_heads, num_pages, page_size,
                 head_dim, dtype, device, page_table=None):
        dimensions = (num_layers, num_kv_heads, num_pages, page_size, head_dim)
        if any(type(size) is not int or size <= 0 for size in dimensions):
            raise ValueError('cache dimensions must be positive integers')
        if dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ValueError('cache dtype must be float32, float16, or bfloat16')
        device = torch.device(device)
        if device.type != 'cuda':
            raise ValueError('paged cache requires a CUDA device')
        page_ids = _checked_page_ids(page_table, num_pages)
        table = torch.tensor(page_ids, dtype=torch.int64, device=device)
        shape = (num_pages, num_kv_heads, page_size, head_dim)
        keys = tuple(torch.empty(shape, dtype=dtype, device=device) for _ in range(num_layers))
        values = tuple(torch.empty(shape, dtype=dtype, device=device) for _ in range(num_layers))
        return cls(keys, values, [0] * num_layers, page_ids, table)

    @property
    def num_layers(self):
        return len(self._keys)

    @property
    def batch_size(self):
        return 1

    @property
    def num_pages(self):
        return self._keys[0].shape[0]

    @property
    def num_kv_heads(self):
        return self._keys[0].shape[1]

    @property
    def page_size(self):
        return self._keys[0].shape[2]

    @property
    def head_dim(self):
        return self._keys[0].shape[3]

    @property
    def page_table(self):
        """Immutable host mapping; the device table stays private."""
        return self._page_ids

    @property
    def capacity(self):
        return len(self._page_ids) * self.page_size

    @property
    def dtype(self):
        return self._keys[0].dtype

    @property
    def device(self):
        return self._keys[0].device

    @property
    def sequence_length(self):
        if any(length != self._lengths[0] for length in self._lengths):
            raise ValueError('cache layers must have aligned lengths before a model call')
        return self._lengths[0]

    def _check_layer(self, layer_idx):
        if type(layer_idx) is not int or not 0 <= layer_idx < self.num_layers:
            raise ValueError('layer index must identify an existing cache layer')

    def length(self, layer_idx):
        self._check_layer(layer_idx)
        return self._lengths[layer_idx]

    def _append_end(self, layer_idx, key, value):
        self._check_layer(layer_idx)
        if not isinstance(key, torch.Tensor) or not isinstance(value, torch.Tensor):
            raise ValueError('keys and values must be tensors')
        if key.layout != torch.strided or value.layout != torch.strided:
            raise ValueError('keys and values must use dense strided storage')
        if (key.ndim != 4 or key.shape != value.shape or key.shape[2] <= 0
                or (key.shape[0], key.shape[1], key.shape[3])
                != (1, self.num_kv_heads, self.head_dim)):
            raise ValueError('K/V must match [1, kv_heads, new_tokens, head_dim] with new_tokens > 0')
        for source in (key, value):
            if source.device != self.device or source.dtype != self.dtype:
                raise ValueError('K/V must match the cache dtype and device')
            if source.requires_grad or source.is_neg():
                raise ValueError('K/V must not require gradients or use lazy negative views')
            if source.stride(-1) != 1 or any(stride < 0 for stride in source.stride()[:-1]):
                raise ValueError('K/V require feature stride 1 and nonnegative outer strides')
            if any(storage_overlaps(source, target)
                   for target in (self._keys[layer_idx], self._values[layer_idx])):
                raise ValueError('K/V inputs must not overlap destination page storage')
        end = self._lengths[layer_idx] + key.shape[2]
        if end > self.capacity:
            raise ValueError('paged KV cache capacity exceeded')
        return end

    @torch.inference_mode()
    def append(self, layer_idx, key, value):
        """Write only new slots; validate predictable failures before any writes."""
        from . import cuda_paged_cache

        end = self._append_end(layer_idx, key, value)
        start = self._lengths[layer_idx]
        cuda_paged_cache._write_paged_kv(key, value, self._keys[layer_idx], self._values[layer_idx],
                                         self._device_page_table, start)
        self._lengths[layer_idx] = end
        return self

    def _gather_buffer(self, pages, length):
        if length == 0:
            return torch.empty((1, self.num_kv_heads, 0, self.head_dim),
                               dtype=self.dtype, device=self.device)
        used = (length + self.page_size - 1) // self.page_size
        ids = self._device_page_table[:used]
        ordered = pages.index_select(0, ids).transpose(0, 1).reshape(
            self.num_kv_heads, used * self.page_size, self.head_dim)
        return ordered[:, :length].unsqueeze(0).contiguous()

    @torch.inference_mode()
    def gather(self, layer_idx):
        """Allocate logical-order K/V copies (tests and checks; decode never gathers)."""
        length = self.length(layer_idx)
        return (self._gather_buffer(self._keys[layer_idx], length),
                self._gather_buffer(self._values[layer_idx], length))

    def reset(self):
        """Clear lengths, preserving physical pages and the fixed mapping."""
        for layer_idx in range(self.num_layers):
            self._lengths[layer_idx] = 0
        return self


class BatchedPagedKVCache:
    """Fixed-page K/V storage for a batch of requests over one shared pool per layer.

    The batched counterpart of ``PagedKVCache`` (the reference caps a cache at
    one request: src/micro_vllm/paged_kv_cache.py:75-77). Per layer, K and V
    pools [num_pages, kv_heads, page_size, head_dim] hold every sequence's
    pages; ``block_table`` [batch, pages_per_seq] (int32, on the device) maps
    each sequence's logical pages to physical ones; ``lengths`` [batch] (int32,
    on the device) counts the tokens each sequence has cached in every layer.
    All sequences advance together (one new token each per decode step), so a
    host copy of the shared length is kept for planning.

    Appends of N tokens for all B sequences are one launch of the paged append
    kernel; the decode step reads the pools in place (``PagedDecodeStep``).
    Lengths advance only through ``advance``, after every layer has appended.
    """

    def __init__(self, keys, values, block_table, lengths, page_size):
        self._keys = tuple(keys)
        self._values = tuple(values)
        self.block_table = block_table
        self.lengths = lengths
        self._length = 0
        self._page_size = page_size

    @classmethod
    def allocate(cls, *, num_layers, batch_size, capacity, num_kv_heads, head_dim, dtype, device,
                 page_size=16, num_pages=None, shuffle_seed=None):
        """Pools for ``batch_size`` sequences of up to ``capacity`` tokens.

        Each sequence owns ceil(capacity / page_size) pages. ``num_pages``
        (default: exactly the pages owned) may add spare pool pages;
        ``shuffle_seed`` scatters the assignment over the pool with a seeded
        permutation, as a fragmented pool would be.
        """
        dims = (num_layers, batch_size, capacity, num_kv_heads, head_dim, page_size)
        if any(type(size) is not int or size <= 0 for size in dims):
            raise ValueError('cache dimensions must be positive integers')
        if dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise ValueError('cache dtype must be float32, float16, or bfloat16')
        device = torch.device(device)
        if device.type != 'cuda':
            raise ValueError('paged cache requires a CUDA device')
        per_seq = (capacity + page_size - 1) // page_size
        needed = batch_size * per_seq
        num_pages = needed if num_pages is None else num_pages
        if type(num_pages) is not int or num_pages < needed:
            raise ValueError('num_pages must cover batch_size * ceil(capacity / page_size)')
        if shuffle_seed is None:
            ids = torch.arange(needed, dtype=torch.int32)
        else:
            gen = torch.Generator().manual_seed(shuffle_seed)
            ids = torch.randperm(num_pages, generator=gen)[:needed].to(torch.int32)
        table = ids.view(batch_size, per_seq).to(device)
        shape = (num_pages, num_kv_heads, page_size, head_dim)
        keys = [torch.empty(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        values = [torch.empty(shape, dtype=dtype, device=device) for _ in range(num_layers)]
        lengths = torch.zeros(batch_size, dtype=torch.int32, device=device)
        return cls(keys, values, table, lengths, page_size)

    @property
    def num_layers(self):
        return len(self._keys)

    @property
    def batch_size(self):
        return self.block_table.shape[0]

    @property
    def num_kv_heads(self):
        return self._keys[0].shape[1]

    @property
    def page_size(self):
        return self._page_size

    @property
    def head_dim(self):
        return self._keys[0].shape[3]

    @property
    def capacity(self):
        return self.block_table.shape[1] * self._page_size

    @property
    def dtype(self):
        return self._keys[0].dtype

    @property
    def device(self):
        return self._keys[0].device

    @property
    def sequence_length(self):
        """Tokens cached per sequence (host copy of the shared length)."""
        return self._length

    def pools(self, layer_idx):
        return self._keys[layer_idx], self._values[layer_idx]

    @torch.inference_mode()
    def append(self, layer_idx, key, value):
        """Write N new tokens of every sequence, [B, Hkv, N, D], at the current lengths."""
        from . import cuda_paged_cache

        if self._length + key.shape[2] > self.capacity:
            raise ValueError('paged KV cache capacity exceeded')
        cuda_paged_cache.write_paged_kv(key, value, self._keys[layer_idx], self._values[layer_idx],
                                        self.block_table, positions=self.lengths)
        return self

    def advance(self, tokens):
        """Count ``tokens`` more cached tokens per sequence (after all layers appended)."""
        if self._length + tokens > self.capacity:
            raise ValueError('paged KV cache capacity exceeded')
        self.lengths += tokens
        self._length += tokens
        return self

    def note_advanced(self, tokens):
        """Host bookkeeping for lengths a captured graph advanced on the device."""
        self._length += tokens
        return self

    @torch.inference_mode()
    def gather(self, layer_idx, sequence, length=None):
        """Logical-order K/V [1, Hkv, L, D] copies of one sequence's first ``length``
        tokens (default: the cached length); tests, checks and chunked prefill."""
        length = self._length if length is None else length
        used = (length + self._page_size - 1) // self._page_size
        ids = self.block_table[sequence, :used].long()

        def ordered(pages):
            rows = pages.index_select(0, ids).transpose(0, 1).reshape(
                self.num_kv_heads, used * self._page_size, self.head_dim)
            return rows[:, :length].unsqueeze(0).contiguous()

        return ordered(self._keys[layer_idx]), ordered(self._values[layer_idx])

    def reset(self):
        self.lengths.zero_()
        self._length = 0
        return self
