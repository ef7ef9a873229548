"""The reference's own CUDA hot-path tests, run against the drop-in API.

Restated from micro-vllm's test/test_cuda_paged_attention.py,
test/test_cuda_paged_cache.py and test/test_paged_attention.py (the
integration part): same inputs, tolerances and error-message patterns, with
``micro_vllm_b200`` in place of ``micro_vllm``. The cache-level tests use the
reference's own ``PagedKVCache`` (installed in baseline/_ref), whose CUDA
append reaches this package through ``integration.install()``. Where the
reference compares against its contiguous-cache kernel (not part of this
path), the fp64 per-head oracle is used instead.
"""
import subprocess
import sys
from pathlib import Path
from unittest.mock import patch

import pytest
import torch

from micro_vllm_b200 import cuda_attention, cuda_paged_cache, integration
from tests.reference_pkg import REF_DIR, reference

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
PagedKVCache = reference('micro_vllm.paged_kv_cache').PagedKVCache


@pytest.fixture(autouse=True)
def reference_routed_here():
    """micro-vllm's native names bound to this package for every test, then restored."""
    with integration.installed():
        yield


def fp64_reference(query, key, value):
    """Per-head fp64 attention of test/test_cuda_gqa.py:14-23, rounded to the query dtype."""
    query_heads, kv_heads = query.shape[1], key.shape[1]
    group = query_heads // kv_heads
    output = torch.empty_like(query, dtype=torch.float64)
    for head in range(query_heads):
        kv_head = head // group
        scores = key[0, kv_head].double() @ query[0, head, 0].double()
        probabilities = torch.softmax(scores * query.shape[-1] ** -0.5, dim=0)
        output[0, head, 0] = probabilities @ value[0, kv_head].double()
    return output.to(query.dtype)


# ------------------------------------------------------------ paged attention

def attention_inputs(length=65, block_size=4, heads=(6, 2), dimension=33, dtype=torch.float32):
    """test/test_cuda_paged_attention.py:20-40: shuffled physical IDs, three pages unassigned,
    every unused slot NaN."""
    hq, hkv = heads
    generator = torch.Generator(device='cuda').manual_seed(519)
    query = torch.randn(1, hq, 1, dimension, dtype=dtype, device='cuda', generator=generator)
    key = torch.randn(1, hkv, length, dimension, dtype=dtype, device='cuda', generator=generator)
    value = torch.randn(key.shape, dtype=dtype, device='cuda', generator=generator)
    count = (length + block_size - 1) // block_size
    ids = list(range(count + 3))[2:count + 2][::-1]
    pages = torch.full((count + 3, hkv, block_size, dimension), float('nan'), dtype=dtype, device='cuda')
    values = torch.full_like(pages, float('nan'))
    for logical, physical in enumerate(ids):
        start, stop = logical * block_size, min((logical + 1) * block_size, length)
        pages[physical, :, :stop - start] = key[0, :, start:stop]
        values[physical, :, :stop - start] = value[0, :, start:stop]
    table = torch.tensor(ids, dtype=torch.int64, device='cuda')
    return query, pages, values, table, key, value


def attend(*args):
    return cuda_attention._load_extension()._decode_attention_paged(*args)


def assert_matches(query, pages, values, table, key, value):
    actual = attend(query, pages, values, table, key.shape[2])
    tolerance = dict(rtol=2e-3, atol=2e-3) if query.dtype == torch.float16 else dict(rtol=2e-4, atol=2e-5)
    torch.testing.assert_close(actual, fp64_reference(query, key, value), **tolerance)
    assert torch.isfinite(actual).all()
    assert actual.is_contiguous()
    assert (actual.shape, actual.dtype, actual.device) == (query.shape, query.dtype, query.device)
    return actual


def test_internal_native_binding_is_available():
    assert hasattr(cuda_attention._load_extension(), '_decode_attention_paged')


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
@pytest.mark.parametrize('block_size', [3, 4, 16, 64])
def test_shuffled_pages_partial_pages_and_tile_boundaries(dtype, block_size):
    for length in sorted({block_size - 1, block_size, block_size + 1, 31, 32, 33, 65, 257}):
        assert_matches(*attention_inputs(length, block_size, dtype=dtype))


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
@pytest.mark.parametrize('heads', [(1, 1), (4, 4), (6, 2), (14, 2), (14, 1)])
@pytest.mark.parametrize('dimension', [33, 257])
def test_generic_gqa_and_feature_tails(dtype, heads, dimension):
    assert_matches(*attention_inputs(heads=heads, dimension=dimension, dtype=dtype))


@pytest.mark.parametrize('dimension', [64, 128])
def test_tensor_core_geometry_through_the_reference_api(dimension):
    """fp16, block 16, D 64/128 takes the TMA + tensor-core kernel."""
    for length in (1, 15, 16, 17, 65, 257, 1025):
        assert_matches(*attention_inputs(length, 16, heads=(14, 2), dimension=dimension,
                                         dtype=torch.float16))


def test_independent_query_strides_including_broadcast_heads():
    query, pages, values, table, key, value = attention_inputs()
    storage = torch.empty(1, 15, 2, 40, device='cuda')
    strided = storage[:, 1:13:2, 1:2, 3:36]
    strided.copy_(query)
    assert not strided.is_contiguous()
    assert_matches(strided, pages, values, table, key, value)
    broadcast = query[:, :1].expand_as(query)
    assert broadcast.stride(1) == 0
    assert_matches(broadcast, pages, values, table, key, value)


def test_inputs_unchanged_outputs_fresh_and_readonly_aliases_allowed():
    query, pages, values, table, key, value = attention_inputs()
    originals = [tensor.clone() for tensor in (query, pages, values, table)]
    first = assert_matches(query, pages, values, table, key, value)
    saved = first.clone()
    second = attend(query, pages, values, table, key.shape[2])
    assert first.data_ptr() != second.data_ptr()
    for tensor, original in zip((query, pages, values, table), originals):
        torch.testing.assert_close(tensor, original, rtol=0, atol=0, equal_nan=True)
        assert first.data_ptr() != tensor.data_ptr()
    torch.testing.assert_close(first, saved, rtol=0, atol=0)
    assert_matches(query, pages, pages, table, key, key)
    alias_query = pages[table[0], :, :1].unsqueeze(0)
    assert_matches(alias_query, pages, pages, table, key, key)


def test_normalized_state_keeps_large_values_finite():
    query, pages, values, table, key, value = attention_inputs()
    query.zero_()
    key.zero_()
    pages.zero_()
    for head, sign in ((0, 1), (1, -1)):
        values[:, head].fill_(sign * 2e38)
        value[:, head].fill_(sign * 2e38)
    actual = attend(query, pages, values, table, key.shape[2])
    assert torch.isfinite(actual).all()
    torch.testing.assert_close(actual, fp64_reference(query, key, value), rtol=5e-6, atol=0)


def test_current_nondefault_stream_orders_table_and_pages():
    query, pages, values, table, key, value = attention_inputs()
    attend(query, pages, values, table, 65)
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        torch.cuda._sleep(10000000)
        query.zero_()
        pages.zero_()
        values.fill_(7)
        table.copy_(table.flip(0))
        actual = attend(query, pages, values, table, 65) * 2
    stream.synchronize()
    torch.testing.assert_close(actual, torch.full_like(query, 14), rtol=2e-5, atol=2e-5)


def test_invalid_used_private_page_ids_cannot_read_out_of_bounds():
    query, pages, values, table, _, _ = attention_inputs()
    for invalid in (-1, pages.shape[0], 2 ** 63 - 1):
        bad_table = table.clone()
        bad_table[8] = invalid  # a later tile must also guard before K/V reads
        actual = attend(query, pages, values, bad_table, 65)
        assert torch.isnan(actual).all()


def test_rejects_invalid_native_metadata_before_launch():
    query, pages, values, table, _, _ = attention_inputs()
    valid = [query, pages, values, table, 65]
    cases = []
    for index, tensor in enumerate(valid[:4]):
        cases.extend([(index, tensor.cpu(), 'CUDA'),
                      (index, torch._neg_view(tensor), 'negative views'),
                      (index, tensor.to_sparse(), 'strided')])
    for index, tensor in enumerate(valid[:3]):
        cases.extend([(index, tensor.double(), 'float32 or float16'),
                      (index, tensor.detach().requires_grad_(), 'gradients')])
    cases.extend([
        (0, query.half(), 'same dtype'), (1, pages.half(), 'same dtype'),
        (2, values.half(), 'same dtype'), (0, query.squeeze(0), 'shape'),
        (0, query.repeat(2, 1, 1, 1), 'batch'),
        (0, query.repeat(1, 1, 2, 1), 'one query'),
        (0, query[:, :0], 'positive'),
        (0, query[:, :3], 'divisible'), (0, query[..., :32], 'head dimension'),
        (0, torch.empty(1, 6, 1, 66, device='cuda')[..., ::2], 'feature stride'),
        (1, pages[:, :, :0].contiguous(), 'positive'),
        (1, pages[:0], 'positive'),
        (1, pages[:, :0].contiguous(), 'positive'),
        (1, pages[..., :0].contiguous(), 'positive'),
        (1, pages[..., :32], 'contiguous'),
        (2, values[:1], 'same shape'),
        (1, pages.squeeze(1).flatten(0, 1), 'shape'),
        (3, table.int(), 'int64'),
        (3, table.unsqueeze(0), 'one-dimensional'),
        (3, table[:0], 'positive'),
        (3, torch.zeros((pages.shape[0] + 1,), device='cuda', dtype=torch.int64), 'physical pages'),
        (3, table.repeat_interleave(2)[::2], 'contiguous'),
        (4, 0, 'positive'), (4, -1, 'positive'),
        (4, table.numel() * pages.shape[2] + 1, 'capacity'),
    ])
    for index, invalid, message in cases:
        args = valid.copy()
        args[index] = invalid
        with pytest.raises(RuntimeError, match=message):
            attend(*args)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason='two CUDA GPUs required')
def test_rejects_mixed_devices_for_every_native_argument():
    query, pages, values, table, _, _ = attention_inputs()
    valid = [query, pages, values, table, 65]
    for index in range(4):
        args = valid.copy()
        args[index] = args[index].to('cuda:1')
        with pytest.raises(RuntimeError, match='same device'):
            attend(*args)


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
@pytest.mark.parametrize('length', [8193, 16385])
def test_no_context_sized_allocations_or_gather_kernels(dtype, length):
    """After the first call the split-KV scratch is cached per stream: a call allocates
    only its output, well under one K row of the context."""
    query, pages, values, table, _, _ = attention_inputs(length, 16, heads=(14, 2), dimension=64,
                                                         dtype=dtype)
    attend(query, pages, values, table, length)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    initial = torch.cuda.memory_allocated()
    actual = attend(query, pages, values, table, length)
    torch.cuda.synchronize()
    peak = torch.cuda.max_memory_allocated() - initial
    assert peak < length * query.element_size()
    assert actual.shape == query.shape


def test_only_this_librarys_kernels_run_in_a_clean_process():
    """test/test_cuda_paged_attention.py:203-233: no gather or copy kernels, only the
    decode kernel (and, when a sequence is split, its merge pass)."""
    script = f'''
import sys
sys.path.insert(0, {str(ROOT / 'micro-vllm_b200')!r})
sys.path.append({str(REF_DIR)!r})
import torch
from micro_vllm_b200 import integration
from micro_vllm_b200.cuda_attention import decode_attention_paged
from micro_vllm.paged_kv_cache import PagedKVCache
integration.install()
cache = PagedKVCache.allocate(
    num_layers=1,num_kv_heads=2,num_pages=5,page_size=32,head_dim=64,
    dtype=torch.float16,device='cuda',page_table=[3,0,2])
q = torch.zeros(1,14,1,64,device='cuda',dtype=torch.float16)
k = torch.zeros(1,2,65,64,device='cuda',dtype=torch.float16)
cache.append(0,k,torch.ones_like(k))
decode_attention_paged(q,cache,layer_idx=0)
torch.cuda.synchronize()
with torch.profiler.profile(activities=[
        torch.profiler.ProfilerActivity.CPU,
        torch.profiler.ProfilerActivity.CUDA]) as profile:
    actual = decode_attention_paged(q,cache,layer_idx=0)
    torch.cuda.synchronize()
kernels = [event.name for event in profile.events()
           if event.device_type == torch.autograd.DeviceType.CUDA]
assert 1 <= len(kernels) <= 2, kernels
assert all('paged_decode' in name for name in kernels), kernels
torch.testing.assert_close(actual,torch.ones_like(q))
print('PAGED_KERNELS_OK', kernels)
'''
    result = subprocess.run([sys.executable, '-c', script], capture_output=True, text=True, timeout=180)
    assert result.returncode == 0, result.stdout + result.stderr
    assert 'PAGED_KERNELS_OK' in result.stdout


# ------------------------------------------------------- public cache-level API

def paged_cache(dtype, length=33, page_size=4):
    needed = (length + page_size - 1) // page_size
    mapping = list(reversed(range(1, needed + 1)))
    return PagedKVCache.allocate(num_layers=2, num_kv_heads=2, num_pages=needed + 2,
                                 page_size=page_size, head_dim=64, dtype=dtype, device='cuda',
                                 page_table=mapping)


@pytest.mark.parametrize('dtype', [torch.float32, torch.float16])
def test_direct_reads_match_per_layer_without_gather(dtype):
    generator = torch.Generator(device='cuda').manual_seed(471)
    cache = paged_cache(dtype)
    for pages in cache._keys + cache._values:
        pages.fill_(float('nan'))
    q = torch.randn(1, 14, 1, 64, device='cuda', dtype=dtype, generator=generator)
    q_saved = q.clone()
    references = []
    for layer, length in ((0, 33), (1, 5)):
        k = torch.randn(1, 2, length, 64, device='cuda', dtype=dtype, generator=generator)
        v = torch.randn(k.shape, device='cuda', dtype=dtype, generator=generator)
        cache.append(layer, k[:, :, :3], v[:, :, :3])
        cache.append(layer, k[:, :, 3:], v[:, :, 3:])
        references.append(fp64_reference(q, k, v))
    snapshots = [p.clone() for p in cache._keys + cache._values]
    with patch.object(cache, 'gather', side_effect=AssertionError('must not gather')), \
            patch.object(cache, '_gather_buffer', side_effect=AssertionError('must not gather')):
        outputs = [cuda_attention.decode_attention_paged(q, cache, layer_idx=layer) for layer in (0, 1)]
    tolerance = dict(rtol=2e-3, atol=2e-3) if dtype == torch.float16 else dict(rtol=2e-4, atol=2e-5)
    for actual, expected in zip(outputs, references):
        torch.testing.assert_close(actual, expected, **tolerance)
        assert actual.shape == q.shape and actual.is_contiguous()
        assert actual.data_ptr() != q.data_ptr()
    torch.testing.assert_close(q, q_saved, rtol=0, atol=0)
    for actual, expected in zip(cache._keys + cache._values, snapshots):
        torch.testing.assert_close(actual, expected, rtol=0, atol=0, equal_nan=True)
    assert (cache.length(0), cache.length(1)) == (33, 5)


def test_reset_and_shorter_reuse_exclude_stale_values():
    cache = paged_cache(torch.float32)
    q = torch.zeros(1, 14, 1, 64, device='cuda')
    cache.append(0, torch.ones(1, 2, 33, 64, device='cuda'), torch.full((1, 2, 33, 64), 99., device='cuda'))
    cuda_attention.decode_attention_paged(q, cache, layer_idx=0)
    cache.reset()
    with pytest.raises(ValueError, match='nonempty'):
        cuda_attention.decode_attention_paged(q, cache, layer_idx=0)
    cache.append(0, torch.zeros(1, 2, 3, 64, device='cuda'), torch.full((1, 2, 3, 64), 7., device='cuda'))
    actual = cuda_attention.decode_attention_paged(q, cache, layer_idx=0)
    torch.testing.assert_close(actual, torch.full_like(q, 7.), rtol=1e-6, atol=1e-6)


def test_workspace_is_output_sized_not_cache_sized():
    cache = paged_cache(torch.float16, length=1025, page_size=16)
    k = torch.zeros(1, 2, 1025, 64, device='cuda', dtype=torch.float16)
    v = torch.ones_like(k)
    cache.append(0, k, v)
    q = torch.zeros(1, 14, 1, 64, device='cuda', dtype=torch.float16)
    cuda_attention.decode_attention_paged(q, cache, layer_idx=0)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    before = torch.cuda.memory_allocated()
    actual = cuda_attention.decode_attention_paged(q, cache, layer_idx=0)
    torch.cuda.synchronize()
    extra = torch.cuda.max_memory_allocated() - before
    assert extra < k.numel() * k.element_size()
    torch.testing.assert_close(actual, torch.ones_like(q), rtol=2e-3, atol=2e-3)


def test_mismatched_query_device_is_rejected():
    cache = paged_cache(torch.float32)
    cache.append(0, torch.zeros(1, 2, 1, 64, device='cuda'), torch.ones(1, 2, 1, 64, device='cuda'))
    with pytest.raises(ValueError, match='device'):
        cuda_attention.decode_attention_paged(torch.zeros(1, 14, 1, 64), cache, layer_idx=0)


# ------------------------------------------------------------------ cache write

def write_arguments(dtype=torch.float32, device='cuda'):
    key = torch.randn((1, 2, 7, 17), dtype=dtype, device=device)
    value = torch.randn_like(key)
    pages = torch.full((5, 2, 4, 17), float('nan'), dtype=dtype, device=device)
    table = torch.tensor([3, 0, 4, 1], dtype=torch.int64, device=device)
    return [key, value, pages, pages.clone(), table, 2]


def assert_exact(actual, expected):
    torch.testing.assert_close(actual, expected, rtol=0, atol=0, equal_nan=True)


def expected_pages(args):
    key, value, key_pages, value_pages, table, start = args
    expected = [key_pages.clone(), value_pages.clone()]
    for token in range(key.size(2)):
        page, slot = divmod(start + token, key_pages.size(2))
        for output, source in zip(expected, (key, value)):
            output[table[page].item(), :, slot, :] = source[0, :, token, :]
    return expected


def assert_write(args):
    original = [tensor.clone() for tensor in args[:2]]
    expected = expected_pages(args)
    pointers = [tensor.data_ptr() for tensor in args[2:4]]
    assert cuda_paged_cache._write_paged_kv(*args) is None
    for output, reference, pointer in zip(args[2:4], expected, pointers):
        assert_exact(output, reference)
        assert output.data_ptr() == pointer
    for source, reference in zip(args[:2], original):
        assert_exact(source, reference)


@pytest.mark.parametrize('dtype', [torch.float16, torch.float32, torch.bfloat16])
def test_write_shuffled_pages_boundaries_dtypes_and_unused_nan(dtype):
    assert_write(write_arguments(dtype))


def test_write_grid_stride_and_odd_feature_dimension():
    key = torch.randn((1, 17, 513, 129), device='cuda')
    pages = torch.full((6, 17, 128, 129), float('nan'), device='cuda')
    args = [key, torch.randn_like(key), pages, pages.clone(),
            torch.tensor([4, 0, 5, 1, 3], device='cuda'), 127]
    assert key.numel() > 4096 * 256
    assert_write(args)


def test_write_chunks_fill_exact_capacity_and_rewrite_after_reset():
    args = write_arguments()
    for start, count in ((0, 3), (3, 5), (8, 8), (0, 1)):
        args[:2] = [torch.randn((1, 2, count, 17), device='cuda') for _ in range(2)]
        args[-1] = start
        assert_write(args)


@pytest.mark.parametrize('dtype', [torch.float16, torch.float32, torch.bfloat16])
def test_write_offset_stepped_and_broadcast_source_strides(dtype):
    args = write_arguments(dtype)
    key = torch.randn((1, 6, 23, 17), device='cuda', dtype=dtype)[:, 1:5:2, 2:23:3]
    value = torch.randn((1, 16, 5, 17), device='cuda', dtype=dtype)[:, 1:15:2, 2:4].transpose(1, 2)
    assert key.stride() != value.stride()
    args[:2] = [key, value]
    assert_write(args)
    args[:2] = [key[:, :1, :1].expand(1, 2, 7, 17), value[:, :1, :1].expand(1, 2, 7, 17)]
    assert_write(args)
    args[1] = args[0]
    assert_write(args)


@pytest.mark.parametrize('dtype, integer', [(torch.float16, torch.int16), (torch.bfloat16, torch.int16),
                                            (torch.float32, torch.int32)])
def test_write_preserves_special_value_bits(dtype, integer):
    args = write_arguments(dtype)
    source = args[0]
    source.flatten()[:4] = torch.tensor([0., -0., float('inf'), -float('inf')], device='cuda')
    payload = 0x7fc12345 if dtype == torch.float32 else (0x7e11 if dtype == torch.float16 else 0x7fc1)
    source.view(integer).flatten()[4] = payload
    args[1] = source
    cuda_paged_cache._write_paged_kv(*args)
    for token in range(source.size(2)):
        page, slot = divmod(args[-1] + token, args[2].size(2))
        for output in args[2:4]:
            assert torch.equal(output[args[4][page], :, slot].view(integer),
                               source[0, :, token].view(integer))


def test_write_current_nondefault_stream():
    stream = torch.cuda.Stream()
    args = write_arguments()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        torch.cuda._sleep(1_000_000)
        args[0].fill_(7.)
        args[1].fill_(-9.)
        cuda_paged_cache._write_paged_kv(*args)
        observed = [tensor.clone() for tensor in args[2:4]]
    stream.synchronize()
    for actual, reference in zip(observed, expected_pages(args)):
        assert_exact(actual, reference)


def assert_rejected(args, message):
    original = [tensor.clone() for tensor in args[2:4]]
    with pytest.raises((RuntimeError, TypeError, ValueError), match=message):
        cuda_paged_cache._write_paged_kv(*args)
    for output, reference in zip(args[2:4], original):
        assert_exact(output, reference)


@pytest.mark.parametrize('index, change, message', [
    (0, lambda x: x.squeeze(0), 'shape'),
    (1, lambda x: x[:, :, :-1], 'shape'),
    (0, lambda x: x.expand(2, -1, -1, -1), 'batch|shape'),
    (0, lambda x: x[:, :, :0], 'positive|shape'),
    (0, lambda x: torch.empty((1, 2, 7, 34), device='cuda')[..., ::2], 'feature stride'),
    (1, lambda x: x.double(), 'dtype'),
    (0, lambda x: x.requires_grad_(), 'gradients'),
    (0, lambda x: torch._neg_view(x), 'negative'),
    (0, lambda x: x.cpu(), 'CUDA'),
    (2, lambda x: x.transpose(0, 2), 'contiguous|shape'),
    (3, lambda x: x[:, :1], 'shape|contiguous'),
    (4, lambda x: x.int(), 'int64'),
    (4, lambda x: x.cpu(), 'CUDA'),
    (4, lambda x: x.reshape(2, 2), '1D|one-dimensional'),
    (4, lambda x: x[:0], 'positive|nonempty'),
    (4, lambda x: torch.arange(6, device='cuda'), 'capacity'),
    (4, lambda x: torch.arange(8, device='cuda')[::2], 'contiguous'),
    (5, lambda x: -1, 'start'),
    (5, lambda x: 10, 'capacity'),
])
def test_write_rejects_invalid_shapes_strides_dtypes_and_capacity(index, change, message):
    args = write_arguments()
    args[index] = change(args[index])
    assert_rejected(args, message)


def test_write_rejects_sparse_and_unsupported_dtypes():
    args = write_arguments()
    args[0] = args[0].to_sparse()
    assert_rejected(args, 'strided')
    args = write_arguments()
    args[:4] = [tensor.to(torch.int32) for tensor in args[:4]]
    assert_rejected(args, 'dtype')


def test_write_rejects_all_source_destination_and_destination_aliases():
    for source in (0, 1):
        for destination in (2, 3):
            args = write_arguments()
            args[source] = args[destination].view(1, 2, 20, 17)[:, :, :7]
            assert_rejected(args, 'alias|storage')
    args = write_arguments()
    args[3] = args[2]
    assert_rejected(args, 'alias|storage')
    args = write_arguments()
    shared = torch.empty(2 * args[2].numel(), device='cuda')
    args[2] = shared[:args[2].numel()].view_as(args[2])
    args[3] = shared[args[2].numel():].view_as(args[3])
    assert_rejected(args, 'alias|storage')


def test_write_rejects_dlpack_aliases_with_independent_storage_metadata():
    for source in (0, 1):
        for destination in (2, 3):
            args = write_arguments()
            view = args[destination].view(1, 2, 20, 17)[:, :, 1:8]
            args[source] = torch.utils.dlpack.from_dlpack(view)
            assert args[source].untyped_storage().data_ptr() != args[destination].untyped_storage().data_ptr()
            assert_rejected(args, 'alias|storage')
    args = write_arguments()
    args[3] = torch.utils.dlpack.from_dlpack(args[2])
    assert_rejected(args, 'alias|storage')
    args = write_arguments()
    table_view = args[2].flatten()[2:10].view(torch.int64)
    args[4] = torch.utils.dlpack.from_dlpack(table_view)
    assert_rejected(args, 'alias|storage')


@pytest.mark.parametrize('dtype', [torch.float16, torch.float32, torch.bfloat16])
def test_high_level_cache_chunks_multilayer_and_reset(dtype):
    """The cache append through the native write agrees with the page-placement rule
    for strided chunks, layer by layer, and reset keeps storage and mapping."""
    options = dict(num_layers=2, num_kv_heads=2, num_pages=5, page_size=4, head_dim=17,
                   dtype=dtype, page_table=[3, 0, 4, 1])
    gpu = PagedKVCache.allocate(**options, device='cuda')
    for pages in (*gpu._keys, *gpu._values):
        pages.fill_(float('nan'))
    buffers = (*gpu._keys, *gpu._values, gpu._device_page_table)
    pointers = [tensor.data_ptr() for tensor in buffers]
    for layer in range(2):
        key = torch.randn((1, 4, 32, 17), device='cuda', dtype=dtype)[:, ::2, ::2]
        value = torch.randn((1, 16, 2, 17), device='cuda', dtype=dtype).transpose(1, 2)
        original = [tensor.clone() for tensor in (key, value)]
        for begin, end in ((0, 3), (3, 8), (8, 16)):
            chunks = (key[:, :, begin:end], value[:, :, begin:end])
            assert gpu.append(layer, *chunks) is gpu
            assert gpu.length(layer) == end
            for actual, expected in zip(gpu.gather(layer), (key[:, :, :end], value[:, :, :end])):
                assert_exact(actual, expected.contiguous())
        for source, saved in zip((key, value), original):
            assert_exact(source, saved)
    assert gpu.sequence_length == 16
    saved = [tensor.clone() for tensor in buffers]
    assert gpu.reset() is gpu
    assert gpu.sequence_length == 0
    for layer in range(2):
        assert gpu.gather(layer)[0].shape == (1, 2, 0, 17)
    for tensor, expected, pointer in zip(buffers, saved, pointers):
        assert_exact(tensor, expected)
        assert tensor.data_ptr() == pointer
    fresh = torch.randn((1, 2, 1, 17), device='cuda', dtype=dtype)
    gpu.append(0, fresh, fresh)
    for actual in gpu.gather(0):
        assert_exact(actual, fresh)
    assert [tensor.data_ptr() for tensor in buffers] == pointers


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason='two CUDA GPUs required')
def test_write_device_mismatch_and_current_device_guard():
    for index in range(5):
        args = write_arguments(device='cuda:0')
        args[index] = args[index].to('cuda:1')
        assert_rejected(args, 'device')
    with torch.cuda.device(1):
        assert_write(write_arguments(device='cuda:0'))
        assert torch.cuda.current_device() == 1
