"""GPU parity of GQA decode over contiguous caches (``decode_attention_gqa``).

Restates the reference's CUDA GQA tests (test/test_cuda_gqa.py,
test_cuda_gqa_strides.py, test_cuda_gqa_precision.py: head ownership, chunk
boundaries, head ratios and feature tails, cache-prefix and strided views,
zero strides, large values, stream order, argument checks) against the fp64
per-head oracle, and checks the batched form on both kernels (tensor-core
split grid via TMA, CUDA-core for the rest) against the same oracle.
"""
import numpy as np
import pytest
import torch

from oracle import decode_fp64_per_head

pytestmark = pytest.mark.gpu


def _api():
    from micro_vllm_b200 import cuda_attention
    return cuda_attention


def fp64(query, key, value):
    """[1,Hq,1,D] / [1,Hkv,L,D] torch -> float64 numpy [Hq, D] (per-head loop)."""
    return decode_fp64_per_head(query[0, :, 0].double().cpu().numpy(), key[0].double().cpu().numpy(),
                                value[0].double().cpu().numpy())


def assert_close(actual, expected, dtype):
    tol = dict(rtol=2e-3, atol=2e-3) if dtype == torch.float16 else (
        dict(rtol=2e-2, atol=2e-2) if dtype == torch.bfloat16 else dict(rtol=2e-4, atol=2e-5))
    np.testing.assert_allclose(actual.double().cpu().numpy(), expected, **tol)


def randn(shape, dtype, gen):
    return torch.randn(shape, generator=gen, device='cuda').to(dtype)


def test_seven_query_heads_share_each_kv_head():
    attention = _api().decode_attention_gqa
    query = torch.zeros(1, 14, 1, 64, device='cuda')
    key = torch.randn(1, 2, 5, 64, device='cuda')
    features = torch.arange(64, device='cuda', dtype=torch.float32)
    value = torch.empty_like(key)
    value[0, 0] = features
    value[0, 1] = features + 1000
    out = attention(query, key, value)
    assert out.shape == query.shape and out.dtype == query.dtype and out.is_contiguous()
    assert torch.allclose(out[0, :7, 0], features.expand(7, 64), atol=1e-5)
    assert torch.allclose(out[0, 7:, 0], (features + 1000).expand(7, 64), atol=1e-3)


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
@pytest.mark.parametrize('length', [1, 15, 16, 17, 31, 32, 33, 65, 257, 1025])
def test_qwen_heads_across_tile_boundaries(dtype, length):
    attention = _api().decode_attention_gqa
    gen = torch.Generator(device='cuda').manual_seed(89 + length)
    query = randn((1, 14, 1, 64), dtype, gen)
    key = randn((1, 2, length, 64), dtype, gen)
    value = randn(key.shape, dtype, gen)
    assert_close(attention(query, key, value)[0, :, 0], fp64(query, key, value), dtype)


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
@pytest.mark.parametrize('heads,dim', [((1, 1), 33), ((4, 4), 64), ((6, 2), 33), ((14, 1), 64),
                                       ((6, 2), 257), ((28, 4), 128), ((32, 2), 256)])
def test_head_ratios_and_feature_tails(dtype, heads, dim):
    attention = _api().decode_attention_gqa
    gen = torch.Generator(device='cuda').manual_seed(101)
    query = randn((1, heads[0], 1, dim), dtype, gen)
    key = randn((1, heads[1], 33, dim), dtype, gen)
    value = randn(key.shape, dtype, gen)
    assert_close(attention(query, key, value)[0, :, 0], fp64(query, key, value), dtype)


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
@pytest.mark.parametrize('length', [31, 32, 33, 65])
def test_cache_prefix_views_skip_unused_capacity(dtype, length):
    """A [1, Hkv, capacity, D] cache read as its [:, :, :length] prefix; NaN past it."""
    attention = _api().decode_attention_gqa
    gen = torch.Generator(device='cuda').manual_seed(617 + length)
    cache_k = torch.full((1, 2, length + 19, 64), float('nan'), dtype=dtype, device='cuda')
    cache_v = torch.full_like(cache_k, float('nan'))
    cache_k[:, :, :length] = randn((1, 2, length, 64), dtype, gen)
    cache_v[:, :, :length] = randn((1, 2, length, 64), dtype, gen)
    key, value = cache_k[:, :, :length], cache_v[:, :, :length]
    assert not key.is_contiguous()
    query = randn((1, 14, 1, 64), dtype, gen)
    before = (cache_k.clone(), cache_v.clone())
    out = attention(query, key, value)
    assert torch.isfinite(out).all()
    assert_close(out[0, :, 0], fp64(query, key, value), dtype)
    assert torch.equal(cache_k.isnan(), before[0].isnan()) and torch.equal(cache_v.isnan(), before[1].isnan())


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
def test_offset_padded_and_stepped_views(dtype):
    attention = _api().decode_attention_gqa
    gen = torch.Generator(device='cuda').manual_seed(7)
    for dim in (64, 257):
        length = 33
        q_store = torch.full((1, 30, 1, dim), 1234., dtype=dtype, device='cuda')
        k_store = torch.full((1, length + 2, 4, dim), 1234., dtype=dtype, device='cuda')
        v_store = torch.full((1, 6, (length + 2) * 3, dim), 1234., dtype=dtype, device='cuda')
        query = q_store[:, 1:29:2]
        key = k_store[:, 1:length + 1, 1:3].transpose(1, 2)
        value = v_store[:, 1:5:2, 2:2 + length * 3:3]
        for t in (query, key, value):
            t.copy_(randn(t.shape, dtype, gen))
        assert_close(attention(query, key, value)[0, :, 0], fp64(query, key, value), dtype)


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
@pytest.mark.parametrize('which', ['query_head', 'key_head', 'value_head', 'key_token', 'value_token',
                                   'unused_outer'])
def test_zero_strides(dtype, which):
    attention = _api().decode_attention_gqa
    gen = torch.Generator(device='cuda').manual_seed(3)
    query = randn((1, 14, 1, 64), dtype, gen)
    key = randn((1, 2, 33, 64), dtype, gen)
    value = randn((1, 2, 33, 64), dtype, gen)
    if which == 'query_head':
        query = randn((1, 1, 1, 64), dtype, gen).expand(1, 14, 1, 64)
    elif which == 'key_head':
        key = randn((1, 1, 33, 64), dtype, gen).expand(1, 2, 33, 64)
    elif which == 'value_head':
        value = randn((1, 1, 33, 64), dtype, gen).expand(1, 2, 33, 64)
    elif which == 'key_token':
        key = randn((1, 2, 1, 64), dtype, gen).expand(1, 2, 33, 64)
    elif which == 'value_token':
        value = randn((1, 2, 1, 64), dtype, gen).expand(1, 2, 33, 64)
    else:
        query = query.as_strided(query.shape, (0, 64, 0, 1))
        key = key.as_strided(key.shape, (0, 33 * 64, 64, 1))
        value = value.as_strided(value.shape, (0, 33 * 64, 64, 1))
    assert_close(attention(query, key, value)[0, :, 0], fp64(query, key, value), dtype)


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
def test_large_values_stay_finite(dtype):
    attention = _api().decode_attention_gqa
    big = 2e38 if dtype == torch.float32 else 60000.0
    query = torch.zeros(1, 14, 1, 64, device='cuda', dtype=dtype)
    key = torch.zeros(1, 2, 65, 64, device='cuda', dtype=dtype)
    value = torch.empty_like(key)
    value[:, 0].fill_(big)
    value[:, 1].fill_(-big)
    out = attention(query, key, value)
    assert torch.isfinite(out).all()
    assert torch.allclose(out[0, :7].float(), torch.full_like(out[0, :7].float(), big), rtol=1e-5)


def test_current_stream_orders_inputs_and_consumers():
    attention = _api().decode_attention_gqa
    query = torch.zeros(1, 14, 1, 64, device='cuda', dtype=torch.float16)
    key = torch.zeros(1, 2, 65, 64, device='cuda', dtype=torch.float16)
    value = torch.zeros_like(key)
    attention(query, key, value)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(10000000)
        query.fill_(1)
        key.fill_(1)
        value[:, 0].fill_(3)
        value[:, 1].fill_(7)
        out = attention(query, key, value) * 2
    stream.synchronize()
    assert (out[:, :7] == 6).all() and (out[:, 7:] == 14).all()


def test_rejects_what_the_reference_rejects():
    attention = _api().decode_attention_gqa
    q = torch.randn(1, 14, 1, 64, device='cuda')
    k = torch.randn(1, 2, 33, 64, device='cuda')
    cases = [
        ((q[..., ::2].contiguous()[..., :32], k, k), 'head dimension'),
        ((torch.randn(1, 14, 1, 128, device='cuda')[..., ::2], k, k), 'feature stride'),
        ((q, torch.randn(1, 2, 33, 128, device='cuda')[..., ::2], k), 'feature stride'),
        ((q.double(), k.double(), k.double()), 'float32 or float16'),
        ((q.half(), k, k), 'same dtype'),
        ((q.expand(2, -1, -1, -1), k.expand(2, -1, -1, -1), k.expand(2, -1, -1, -1)), 'batch size 1'),
        ((torch.randn(1, 14, 2, 64, device='cuda'), k, k), 'one query token'),
        ((q[:, :13], k, k), 'divisible'),
        ((q, k, k[:, :, :5]), 'same shape'),
        ((q.cpu(), k, k), 'CUDA'),
    ]
    for args, message in cases:
        with pytest.raises(RuntimeError, match=message):
            attention(*args)


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize('mode', [{}, dict(force_simt=True), dict(wide=True), dict(pages_per_split=2)])
def test_batched_prefix_views_per_sequence_lengths(dtype, mode):
    """[B, Hkv, capacity, D] caches, per-sequence device lengths, every kernel."""
    api = _api()
    gen = torch.Generator(device='cuda').manual_seed(11)
    batch, hq, hkv, dim, cap = 5, 28, 4, 128, 300
    k_store = randn((batch, hkv, cap + 8, dim), dtype, gen)
    v_store = randn((batch, hkv, cap + 8, dim), dtype, gen)
    key, value = k_store[:, :, :cap], v_store[:, :, :cap]
    query = randn((batch, hq, dim), dtype, gen)
    lens = torch.tensor([1, 16, 17, 255, 300], dtype=torch.int32, device='cuda')
    out = api.contiguous_decode_attention(query, key, value, lens, **mode)
    path = api.contiguous_decode_plan(key, value, hq, **mode)[0]
    assert path == ('simt' if mode.get('force_simt') or dtype == torch.float32 else 'tma_mma')
    for b, length in enumerate(lens.tolist()):
        expected = decode_fp64_per_head(query[b].double().cpu().numpy(),
                                        key[b, :, :length].double().cpu().numpy(),
                                        value[b, :, :length].double().cpu().numpy())
        assert_close(out[b], expected, dtype)


def test_batched_lengths_above_the_bound_are_nan_and_zero_length_is_zero():
    api = _api()
    gen = torch.Generator(device='cuda').manual_seed(12)
    key = randn((3, 2, 64, 128), torch.bfloat16, gen)
    value = randn((3, 2, 64, 128), torch.bfloat16, gen)
    query = randn((3, 14, 128), torch.bfloat16, gen)
    lens = torch.tensor([0, 64, 65], dtype=torch.int64, device='cuda')
    for mode in ({}, dict(force_simt=True)):
        out = api.contiguous_decode_attention(query, key, value, lens, **mode).float()
        assert (out[0] == 0).all() and torch.isfinite(out[1]).all() and torch.isnan(out[2]).all()


def test_unaligned_cache_views_take_the_cuda_core_kernel():
    api = _api()
    gen = torch.Generator(device='cuda').manual_seed(13)
    store = randn((2, 2, 40, 129), torch.bfloat16, gen)
    key = store[..., 1:]        # base 2 bytes off 16, rows of 258 bytes
    value = store[..., :128]
    query = randn((2, 8, 128), torch.bfloat16, gen)
    assert api.contiguous_decode_plan(key, value, 8)[0] == 'simt'
    out = api.contiguous_decode_attention(query, key, value)
    for b in range(2):
        assert_close(out[b], decode_fp64_per_head(query[b].double().cpu().numpy(), key[b].double().cpu().numpy(),
                                                  value[b].double().cpu().numpy()), torch.bfloat16)


def test_multi_wave_grid_with_a_first_split_matches_the_oracle():
    """A batch big enough for more than one wave of CTAs takes the first-split
    schedule (split 0 twice the split size, split-major order) on contiguous
    caches too; checked against the fp64 oracle on a sample of sequences, and
    against the uniform-split plan of the same size on all of them."""
    api = _api()
    gen = torch.Generator(device='cuda').manual_seed(21)
    batch, hq, hkv, dim, cap = 128, 28, 4, 128, 704
    key = randn((batch, hkv, cap, dim), torch.bfloat16, gen)
    value = randn((batch, hkv, cap, dim), torch.bfloat16, gen)
    query = randn((batch, hq, dim), torch.bfloat16, gen)
    lens = torch.randint(1, cap + 1, (batch,), generator=torch.Generator().manual_seed(22)).to(torch.int32).cuda()
    path, pps, splits = api.contiguous_decode_plan(key, value, hq)
    max_pages = cap // 16
    assert path == 'tma_mma' and 2 * pps < max_pages
    assert splits == 1 + -(-(max_pages - 2 * pps) // pps)      # a first split of 2 x pps runs
    out = api.contiguous_decode_attention(query, key, value, lens)
    uniform = api.contiguous_decode_attention(query, key, value, lens, pages_per_split=pps)
    np.testing.assert_allclose(out.float().cpu().numpy(), uniform.float().cpu().numpy(), rtol=2e-2, atol=2e-2)
    for b in range(0, batch, 9):
        length = int(lens[b])
        expected = decode_fp64_per_head(query[b].double().cpu().numpy(),
                                        key[b, :, :length].double().cpu().numpy(),
                                        value[b, :, :length].double().cpu().numpy())
        assert_close(out[b], expected, torch.bfloat16)
