"""Host-side checks of the reference-shaped API, run before any native code loads.

Restates the reference's CPU tests for the public paged decode entry point
(test/test_paged_attention.py:14-89): foreign caches, bad layers, empty
layers, malformed queries and non-CUDA caches are rejected with ValueError
before the extension is loaded, and nothing is gathered. The caches are the
reference's own ``PagedKVCache`` (installed in baseline/_ref), the object the
drop-in receives from micro-vllm's model code.
"""
from unittest.mock import patch

import pytest
import torch

from micro_vllm_b200 import cuda_attention, cuda_paged_cache
from tests.reference_pkg import reference


def cpu_cache(dtype=torch.float32):
    """The reference's cache over CPU tensors, built through its dataclass constructor."""
    PagedKVCache = reference('micro_vllm.paged_kv_cache').PagedKVCache
    keys = tuple(torch.zeros(7, 2, 4, 8, dtype=dtype) for _ in range(2))
    values = tuple(torch.zeros(7, 2, 4, 8, dtype=dtype) for _ in range(2))
    return PagedKVCache(keys, values, [5, 0], (4, 1, 5), torch.tensor([4, 1, 5]))


class ContiguousLike:
    """Stands in for a non-paged cache type."""

    def length(self, layer_idx):
        return 1


def test_rejects_foreign_cache_types_before_loading():
    q = torch.zeros(1, 4, 1, 8)
    with patch.object(cuda_attention, '_load_extension') as load:
        for cache in (None, ContiguousLike(), object()):
            with pytest.raises(ValueError, match='PagedKVCache'):
                cuda_attention.decode_attention_paged(q, cache, layer_idx=0)
        load.assert_not_called()


def test_layer_and_empty_cache_rejection_preserve_lengths():
    cache = cpu_cache()
    q = torch.zeros(1, 4, 1, 8)
    with patch.object(cuda_attention, '_load_extension') as load:
        for layer in (-1, 2, True, 1.5, None):
            with pytest.raises(ValueError, match='layer'):
                cuda_attention.decode_attention_paged(q, cache, layer_idx=layer)
        with pytest.raises(ValueError, match='nonempty'):
            cuda_attention.decode_attention_paged(q, cache, layer_idx=1)
        load.assert_not_called()
    assert (cache.length(0), cache.length(1)) == (5, 0)


@pytest.mark.parametrize('make, message', [
    (lambda q: None, 'tensor'),
    (lambda q: q.to_sparse(), 'strided'),
    (lambda q: q[0], 'shape'),
    (lambda q: q.expand(2, -1, -1, -1), 'shape'),
    (lambda q: q.expand(-1, -1, 2, -1), 'shape'),
    (lambda q: q[:, :0], 'shape'),
    (lambda q: q[..., :7], 'shape'),
    (lambda q: q[:, :3], 'divisible'),
    (lambda q: q.half(), 'dtype'),
    (lambda q: q.double(), 'dtype'),
    (lambda q: q.detach().requires_grad_(), 'gradients'),
    (lambda q: torch._neg_view(q), 'negative'),
    (lambda q: torch.zeros(1, 4, 1, 16)[..., ::2], 'feature stride'),
])
def test_query_formats_fail_before_loading(make, message):
    cache = cpu_cache()
    with patch.object(cuda_attention, '_load_extension') as load:
        with pytest.raises(ValueError, match=message):
            cuda_attention.decode_attention_paged(make(torch.zeros(1, 4, 1, 8)), cache, layer_idx=0)
        load.assert_not_called()


def test_cpu_cache_is_not_gathered_or_run_on_the_host():
    cache = cpu_cache()
    with patch.object(cache, 'gather', side_effect=AssertionError('must not gather')), \
            patch.object(cuda_attention, '_load_extension') as load:
        with pytest.raises(ValueError, match='CUDA'):
            cuda_attention.decode_attention_paged(torch.zeros(1, 4, 1, 8), cache, layer_idx=0)
        load.assert_not_called()


def test_bfloat16_is_rejected_like_the_reference():
    cache = cpu_cache(torch.bfloat16)
    with pytest.raises(ValueError, match='float16 or float32'):
        cuda_attention.decode_attention_paged(torch.zeros(1, 4, 1, 8, dtype=torch.bfloat16), cache,
                                              layer_idx=0)


def test_native_write_checks_name_cuda_first():
    """The write's native-level checks (paged_kv_cache.cpp:19-24) start with the device."""
    key = torch.zeros(1, 2, 3, 8)
    pages = torch.zeros(4, 2, 4, 8)
    table = torch.tensor([0, 1])
    with patch.object(cuda_paged_cache._native, 'library') as lib:
        with pytest.raises(RuntimeError, match='CUDA'):
            cuda_paged_cache._PagedCacheExtension().write_paged_kv(key, key, pages, pages.clone(),
                                                                   table, 0)
        lib.assert_not_called()


def test_native_decode_checks_name_cuda_first():
    q = torch.zeros(1, 4, 1, 8)
    pages = torch.zeros(4, 2, 4, 8)
    table = torch.tensor([0, 1])
    with patch.object(cuda_attention._native, 'library') as lib:
        with pytest.raises(RuntimeError, match='CUDA'):
            cuda_attention._DecodeAttentionExtension()._decode_attention_paged(q, pages, pages, table, 5)
        lib.assert_not_called()


def test_batched_step_checks_run_before_loading():
    """The one-call append + attend step validates on the host before any native call."""
    q = torch.zeros(2, 4, 8)
    rows = torch.zeros(2, 2, 8)
    pages = torch.zeros(4, 2, 16, 8)
    table = torch.zeros(2, 2, dtype=torch.int32)
    lens = torch.ones(2, dtype=torch.int32)
    with patch.object(cuda_attention._native, 'library') as lib:
        with pytest.raises(RuntimeError, match='CUDA'):
            cuda_attention.paged_decode_with_append(q, rows, rows, pages, pages.clone(), table, lens)
        lib.assert_not_called()


def test_storage_overlap_detects_views_and_dlpack_aliases():
    from micro_vllm_b200._tensors import storage_overlaps
    base = torch.zeros(64)
    assert storage_overlaps(base[:10], base[5:20])
    assert storage_overlaps(base[:4], base[60:])  # same storage, any offsets
    assert not storage_overlaps(base, torch.zeros(64))
    alias = torch.utils.dlpack.from_dlpack(base[8:16])
    assert storage_overlaps(alias, base)
    assert not storage_overlaps(torch.zeros(0), base)


def test_batched_cache_and_runtime_refuse_cpu_storage():
    from micro_vllm_b200.paged_kv_cache import BatchedPagedKVCache
    from micro_vllm_b200.runtime import prepare_model
    from tests.golden.model_cases import make_weights, model_config
    with pytest.raises(ValueError, match='CUDA'):
        BatchedPagedKVCache.allocate(num_layers=1, batch_size=2, capacity=32, num_kv_heads=1, head_dim=8,
                                     dtype=torch.float32, device='cpu')
    with pytest.raises(ValueError, match='positive integers'):
        BatchedPagedKVCache.allocate(num_layers=1, batch_size=0, capacity=32, num_kv_heads=1, head_dim=8,
                                     dtype=torch.float32, device='cuda')
    weights = {k: torch.from_numpy(v) for k, v in make_weights('tiny_qwen2_fp32').items()}
    with pytest.raises(ValueError, match='CUDA weights'):
        prepare_model(weights, model_config('tiny_qwen2_fp32'))


def test_generate_rejects_bad_arguments_before_any_work():
    from micro_vllm_b200.generate import _eos_ids, greedy_decode
    with pytest.raises(ValueError, match='max_new_tokens'):
        greedy_decode({}, None, torch.zeros(1, 4, dtype=torch.long), 0)
    with pytest.raises(ValueError, match='equal-length prompts'):
        greedy_decode({}, None, torch.zeros(4, dtype=torch.long), 2)
    assert _eos_ids(None, 10) == () and _eos_ids(3, 10) == (3,) and _eos_ids([1, 2], 10) == (1, 2)
    with pytest.raises(ValueError, match='EOS'):
        _eos_ids(11, 10)
