"""micro-vllm's own model code and cache, running this package's kernels.

Restates micro-vllm's paged-forward GPU tests (test/test_paged_forward.py:120-163)
with ``micro_vllm_b200.integration.install()`` in effect: the reference's
``PreparedModel.forward`` drives its own ``PagedKVCache`` through the call site
of model.py:170-182, appending before attending (model.py:215-216), and the
native names it calls -- ``model.decode_attention_paged``,
``cuda_paged_cache._write_paged_kv`` and, for the contiguous cache,
``cuda_attention.decode_attention_gqa`` -- are this package's. The
reference's JIT-built extensions must never load.

As in the reference test: four forwards (a 3-token prefill, then three
single-token decodes) over a NaN-poisoned paged cache with 3-token pages and
the page table (4, 1, 5, 0); exactly 3 x layers paged decodes, 4 x layers cache
writes, one attention_forward per layer (the prefill) and no gather; then the
logits and the stored K/V against the contiguous-cache path. The reference
asserts bit equality there because both of its caches run one kernel; here
the paged decode (3-token pages) and the contiguous decode can take different
kernels of this package (the CUDA-core kernel for odd page sizes, the
tensor-core tile for 16-byte aligned contiguous fp16 caches), so logits are
held to the parity bar of the dtype, and the first layer's stored K/V -- which
no attention output feeds -- to bit equality.
"""
from unittest.mock import patch

import pytest
import torch

from micro_vllm_b200 import cuda_attention, cuda_paged_cache, integration
from tests.golden.model_cases import CALL_SITE_CONFIG, config_object, weights_for
from tests.reference_pkg import reference

pytestmark = pytest.mark.gpu

CHUNKS = ((0, 3), (3, 4), (4, 5), (5, 6))
TOLERANCE = {torch.float32: dict(rtol=1e-5, atol=1e-6), torch.float16: dict(rtol=2e-3, atol=2e-3)}


def _model(dtype):
    config = config_object(CALL_SITE_CONFIG)
    weights = {name: torch.from_numpy(array).to(device='cuda', dtype=dtype)
               for name, array in weights_for(CALL_SITE_CONFIG, 123, 0.02).items()}
    return config, weights


def _paged(config, dtype, page_size=3, mapping=(4, 1, 5, 0)):
    PagedKVCache = reference('micro_vllm.paged_kv_cache').PagedKVCache
    head_dim = config.hidden_size // config.num_attention_heads
    cache = PagedKVCache.allocate(num_layers=config.num_hidden_layers, num_kv_heads=config.num_key_value_heads,
                                  num_pages=max(mapping) + 2, page_size=page_size, head_dim=head_dim,
                                  dtype=dtype, device='cuda', page_table=mapping)
    for tensor in cache._keys + cache._values:
        tensor.fill_(float('nan'))
    return cache


def _dense(config, dtype, capacity):
    ContiguousKVCache = reference('micro_vllm.kv_cache').ContiguousKVCache
    return ContiguousKVCache.allocate(num_layers=config.num_hidden_layers, batch_size=1,
                                      num_kv_heads=config.num_key_value_heads, capacity=capacity,
                                      head_dim=config.hidden_size // config.num_attention_heads,
                                      dtype=dtype, device='cuda')


def _no_reference_extensions():
    ref_attention = reference('micro_vllm.cuda_attention')
    ref_cache = reference('micro_vllm.cuda_paged_cache')
    return (patch.object(ref_attention, '_load_extension',
                         side_effect=AssertionError('reference attention extension must not load')),
            patch.object(ref_cache, '_load_extension',
                         side_effect=AssertionError('reference cache extension must not load')))


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
@pytest.mark.parametrize('mode', ['auto', 'cuda'])
def test_full_optimized_path_has_no_gather_and_uses_this_packages_operators(dtype, mode):
    model = reference('micro_vllm.model')
    ref_cache = reference('micro_vllm.cuda_paged_cache')
    config, weights = _model(dtype)
    layers = config.num_hidden_layers
    ids = torch.tensor([[10, 20, 30, 40, 50, 60]], device='cuda')
    no_attention_ext, no_cache_ext = _no_reference_extensions()
    with integration.installed(), no_attention_ext, no_cache_ext:
        assert model.decode_attention_paged is cuda_attention.decode_attention_paged
        assert ref_cache._write_paged_kv is cuda_paged_cache._write_paged_kv
        prepared = model.prepare_model(weights, config, attention_backend=mode)
        paged, dense = _paged(config, dtype), _dense(config, dtype, capacity=12)
        outputs = []
        with patch.object(paged, 'gather', side_effect=AssertionError('must not gather')), \
                patch.object(model, 'decode_attention_paged', wraps=model.decode_attention_paged) as decode, \
                patch.object(ref_cache, '_write_paged_kv', wraps=ref_cache._write_paged_kv) as write, \
                patch.object(model, 'attention_forward', wraps=model.attention_forward) as attention:
            for start, end in CHUNKS:
                outputs.append(prepared.forward(ids[:, start:end], cache=paged))
            assert decode.call_count == 3 * layers
            assert write.call_count == 4 * layers
            assert attention.call_count == layers
            expected_route = 'flash' if mode == 'auto' and dtype == torch.float16 else 'torch'
            assert all(call.kwargs['implementation'] == expected_route for call in attention.call_args_list)
        expected = [prepared.forward(ids[:, a:b], cache=dense) for a, b in CHUNKS]
        torch.cuda.synchronize()
    actual, expected = torch.cat(outputs, 1), torch.cat(expected, 1)
    assert torch.isfinite(actual).all()
    torch.testing.assert_close(actual, expected, **TOLERANCE[dtype])
    assert paged.sequence_length == 6
    for layer in range(layers):
        for left, right in zip(paged.gather(layer), dense.read(layer)):
            if layer == 0:
                assert torch.equal(left, right)
            else:
                torch.testing.assert_close(left, right, **TOLERANCE[dtype])


def test_cached_multi_token_chunk_keeps_the_reference_fallback():
    """A cached chunk of several tokens gathers and runs the reference's attention,
    with this package's cache write; logits match the contiguous cache (within the
    fp16 bar: the single-token steps between chunks run this package's decode)."""
    model = reference('micro_vllm.model')
    config, weights = _model(torch.float16)
    no_attention_ext, no_cache_ext = _no_reference_extensions()
    with integration.installed(), no_attention_ext, no_cache_ext:
        prepared = model.prepare_model(weights, config)
        paged, dense = _paged(config, torch.float16, page_size=2), _dense(config, torch.float16, capacity=8)
        ids = torch.tensor([[10, 20, 30, 40, 50, 60, 70]], device='cuda')
        offset = 0
        for count in (2, 1, 3, 1):
            chunk = ids[:, offset:offset + count]
            left = prepared.forward(chunk, cache=paged)
            right = prepared.forward(chunk, cache=dense)
            torch.testing.assert_close(left, right, **TOLERANCE[torch.float16])
            offset += count
