"""Fixed-page K/V storage for a batch of requests over one shared page pool.

micro-vllm's own ``PagedKVCache`` (src/micro_vllm/paged_kv_cache.py:43-199)
holds one request; the drop-in decode path reads that class as it is
(``cuda_attention.decode_attention_paged`` takes the reference's cache object
and reads its ``_keys``, ``_values``, ``_device_page_table`` and ``length``),
and its CUDA append reaches this package through
``cuda_paged_cache._write_paged_kv`` (see ``integration``). This module adds
the batched cache the batched runtime and serving loop need: one pool per
layer shared by every sequence, a device block table and device lengths, the
same page layout [num_pages, kv_heads, page_size, head_dim].
"""
import torch


class BatchedPagedKVCache:
    """Fixed-page K/V storage for a batch of requests over one shared pool per layer.

    The batched counterpart of micro-vllm's ``PagedKVCache``, which caps a
    cache at one request (src/micro_vllm/paged_kv_cache.py:75-77). Per layer, K and V
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
