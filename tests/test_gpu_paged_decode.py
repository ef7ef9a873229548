"""GPU parity: append + paged decode through the C ABI against the CPU oracle.

Every case regenerates the seeded inputs, appends the step's token with the
batched append kernel, checks the pools bit-for-bit against the digests the
reference's own code produced (tests/golden/), then checks attention against
the oracle at the parity bar (fp32 1e-5 relative, fp16 2e-3, bf16 2e-2 max-abs
of the fp32 math), on both kernels and with forced split-KV.
"""
import numpy as np
import pytest
import torch

from oracle import decode_float, decode_fp64_per_head, to_float32
from tests.golden.cases import array_digest, make_inputs
from tests.golden.make_golden import GOLDEN_CASES
from tests.helpers import as_float, assert_attention_close, to_numpy, to_torch, workload_tensors

pytestmark = pytest.mark.gpu


def _native():
    from micro_vllm_b200 import cuda_attention, cuda_paged_cache
    return cuda_attention, cuda_paged_cache


def _fixture(name):
    from pathlib import Path
    with np.load(Path(__file__).resolve().parent / 'golden' / f'{name}.npz') as data:
        return {key: data[key] for key in data.files}


def _append_and_decode(inputs, **mode):
    attention, cache = _native()
    t = workload_tensors(inputs)
    cache.write_paged_kv(t['key_new'], t['value_new'], t['key_pool'], t['value_pool'],
                         t['block_table'], positions=t['context_lens'], positions_are_end=True)
    out = attention.paged_decode_attention(
        t['q'], t['key_pool'], t['value_pool'], t['block_table'], t['context_lens'], **mode)
    torch.cuda.synchronize()
    return t, out


def _oracle(inputs, key_pool, value_pool):
    dim = inputs['q'].shape[-1]
    return decode_float(inputs['q'], key_pool, value_pool, inputs['block_table'],
                        inputs['context_lens'], dim ** -0.5, inputs['spec']['dtype'])


MODES = {
    'auto': {},                               # tensor-core split grid + merge pass
    'cluster': dict(cluster=True),            # tensor-core cluster kernel (contexts up to 8192 tokens)
    'persistent': dict(persistent=True),      # tensor-core persistent schedule + merge pass
    'fused': dict(fused_merge=True),          # split grid, last split CTA merges
    'split4': dict(pages_per_split=4),        # split grid, 4 pages per split
    'wide': dict(wide=True),                  # split grid, wide shape (8 warps, deeper rings)
    'simt': dict(force_simt=True),            # CUDA-core kernel
    'cuda_core_math': dict(cuda_core_math=True),  # split grid, fp32 FMA math (group <= 8, D 64/128)
}


@pytest.mark.parametrize('name', GOLDEN_CASES)
@pytest.mark.parametrize('mode', list(MODES))
def test_golden_workloads(name, mode):
    inputs = make_inputs(name)
    dtype = inputs['spec']['dtype']
    t, out = _append_and_decode(inputs, **MODES[mode])
    fixture = _fixture(name)
    key_pool = to_numpy(t['key_pool'])
    value_pool = to_numpy(t['value_pool'])
    # The append is bit-exact against the pools the reference's own append produced.
    assert array_digest(key_pool) == str(fixture['key_pool_digest'])
    assert array_digest(value_pool) == str(fixture['value_pool_digest'])
    expected = _oracle(inputs, key_pool, value_pool)
    assert_attention_close(as_float(out), expected, dtype)
    # And close to the reference's own output within its own dtype rounding.
    reference = to_float32(fixture['out'], dtype)
    bound = {'float32': 2e-5, 'float16': 4e-3, 'bfloat16': 0.15}[dtype]
    assert np.max(np.abs(as_float(out) - reference)) <= bound


def test_tensor_core_paths_are_selected_for_qwen_geometry():
    attention, _ = _native()
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    path, pps, splits = attention.paged_decode_plan(28, t['key_pool'], 4096, batch=64)
    assert path == 'tma_mma' and splits >= 2
    path, pps, splits = attention.paged_decode_plan(28, t['key_pool'], 4096, batch=64, cluster=True)
    assert path == 'tma_mma_cluster' and pps <= 64
    assert attention.paged_decode_plan(28, t['key_pool'], 32768, batch=8, cluster=True)[0] == 'tma_mma'
    assert attention.paged_decode_plan(28, t['key_pool'], 4096, batch=64, persistent=True)[0] == \
        'tma_mma_persistent'
    assert attention.paged_decode_plan(28, t['key_pool'], 4096, batch=64, force_simt=True)[0] == 'simt'
    assert attention.paged_decode_plan(28, t['key_pool'].float(), 4096, batch=64)[0] == 'simt'


@pytest.mark.parametrize('lens', [[1], [16], [17], [1, 1, 1], [4096, 1, 33], [5000, 40, 7, 0, 3000],
                                  [16] * 37, [1029, 700, 1] * 5])
def test_persistent_ranges_cover_every_length_mix(lens):
    """Equal page ranges per warp cut segments anywhere; check many length mixes."""
    spec = dict(batch=len(lens), q_heads=28, kv_heads=4, head_dim=128, block_size=16,
                pool=('factor', 1.3), lens=('fixed', lens), dtype='bfloat16', value_scale=0.5,
                seed=31 + len(lens))
    inputs = make_inputs(spec)
    for mode in ('auto', 'cluster', 'persistent'):
        t, out = _append_and_decode(inputs, **MODES[mode])
        expected = _oracle(inputs, to_numpy(t['key_pool']), to_numpy(t['value_pool']))
        assert_attention_close(as_float(out), expected, 'bfloat16')


@pytest.mark.parametrize('max_len', [16, 64, 65, 128, 129, 300, 1024, 2047, 4096, 8192])
def test_cluster_sizes_cover_every_bound(max_len):
    """The cluster kernel splits each sequence over 1..8 CTAs by the host bound;
    lengths well under the bound leave CTAs of a cluster with no pages."""
    lens = sorted({1, max(1, max_len // 3), max_len})
    spec = dict(batch=len(lens), q_heads=28, kv_heads=4, head_dim=128, block_size=16,
                pool=('factor', 1.2), lens=('fixed', lens), dtype='bfloat16', value_scale=0.5,
                seed=max_len)
    inputs = make_inputs(spec)
    attention, cache = _native()
    t = workload_tensors(inputs)
    cache.write_paged_kv(t['key_new'], t['value_new'], t['key_pool'], t['value_pool'],
                         t['block_table'], positions=t['context_lens'], positions_are_end=True)
    assert attention.paged_decode_plan(28, t['key_pool'], max_len, batch=len(lens),
                                       cluster=True)[0] == 'tma_mma_cluster'
    out = attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], t['block_table'],
                                           t['context_lens'], max_context_len=max_len, cluster=True)
    expected = _oracle(inputs, to_numpy(t['key_pool']), to_numpy(t['value_pool']))
    assert_attention_close(as_float(out), expected, 'bfloat16')


def test_workspace_counters_reset_across_calls_and_paths():
    """The fused split merge counts arrivals in the shared workspace; alternating
    kernels and shapes on one stream must keep giving identical results."""
    attention, _ = _native()
    small = workload_tensors(make_inputs('qwen7b_bf16_small'))
    big = workload_tensors(make_inputs('qwen72b_bf16_small'))
    runs = []
    for _ in range(3):
        row = []
        for t in (small, big):
            for mode in MODES.values():
                row.append(attention.paged_decode_attention(
                    t['q'], t['key_pool'], t['value_pool'], t['block_table'], t['context_lens'],
                    **mode).clone())
        runs.append(row)
    for row in runs[1:]:
        for a, b in zip(runs[0], row):
            assert torch.equal(a, b)


@pytest.mark.parametrize('pages_per_split', [1, 4, 8, 12, 128])
def test_split_counts_agree(pages_per_split):
    inputs = make_inputs('qwen7b_bf16_small')
    _, reference_out = _append_and_decode(inputs, pages_per_split=128)
    inputs = make_inputs('qwen7b_bf16_small')
    t, out = _append_and_decode(inputs, pages_per_split=pages_per_split)
    expected = _oracle(inputs, to_numpy(t['key_pool']), to_numpy(t['value_pool']))
    assert_attention_close(as_float(out), expected, 'bfloat16')
    assert np.max(np.abs(as_float(out) - as_float(reference_out))) <= 1e-2


@pytest.mark.parametrize('name', ['qwen7b_bf16_small', 'qwen05b_fp32', 'edge_bs4_d257_fp16'])
def test_invalid_page_id_poisons_only_that_sequence(name):
    attention, _ = _native()
    inputs = make_inputs(name)
    spec = inputs['spec']
    t = workload_tensors(inputs)
    lens = inputs['context_lens']
    victim = int(np.argmax(lens))
    used = -(-int(lens[victim]) // spec['block_size'])
    for bad in (-1, t['key_pool'].shape[0], 2 ** 31 - 1):
        table = t['block_table'].clone()
        table[victim, used - 1] = bad
        for mode in MODES.values():
            out = attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], table,
                                                   t['context_lens'], **mode)
            values = as_float(out)
            assert np.isnan(values[victim]).all()
            others = np.delete(values, victim, axis=0)
            assert np.isfinite(others).all()


def test_zero_and_out_of_range_lengths():
    attention, _ = _native()
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    capacity = t['block_table'].shape[1] * 16
    lens = t['context_lens'].clone()
    lens[0] = 0
    lens[1] = capacity + 1
    lens[2] = -5
    for mode in MODES.values():
        out = as_float(attention.paged_decode_attention(
            t['q'], t['key_pool'], t['value_pool'], t['block_table'], lens, **mode))
        assert (out[0] == 0).all()
        assert np.isnan(out[1]).all() and np.isnan(out[2]).all()


def test_lengths_above_the_planned_bound_are_nan_not_out_of_bounds():
    attention, _ = _native()
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    out = as_float(attention.paged_decode_attention(
        t['q'], t['key_pool'], t['value_pool'], t['block_table'], t['context_lens'],
        max_context_len=100))
    lens = inputs['context_lens']
    assert np.isnan(out[lens > 100]).all()
    assert np.isfinite(out[lens <= 100]).all()


@pytest.mark.parametrize('dtype', ['bfloat16', 'float16', 'float32'])
def test_nan_in_unused_slots_does_not_leak(dtype):
    """Slots past the context in the last page are NaN; P*V must not see them."""
    attention, _ = _native()
    spec = dict(make_inputs('qwen7b_bf16_small')['spec'])
    spec.update(dtype=dtype, lens=('fixed', [5, 33, 47]), seed=77)
    inputs = make_inputs(spec)
    t = workload_tensors(inputs)
    bs = spec['block_size']
    lens = inputs['context_lens']
    for b in range(spec['batch']):
        last = int(inputs['block_table'][b, (lens[b] - 1) // bs])
        slot = int(lens[b] % bs)
        if slot:
            t['key_pool'][last, :, slot:] = float('nan')
            t['value_pool'][last, :, slot:] = float('nan')
    for mode in MODES.values():
        out = attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'],
                                               t['block_table'], t['context_lens'], **mode)
        expected = _oracle(inputs, to_numpy(t['key_pool']), to_numpy(t['value_pool']))
        assert np.isfinite(as_float(out)).all()
        assert_attention_close(as_float(out), expected, dtype)


@pytest.mark.parametrize('dtype', [torch.float16, torch.bfloat16])
def test_large_logits_pick_the_argmax_value_exactly(dtype):
    """test/test_cuda_gqa_precision.py:92-102 on pages: a one-hot softmax returns V exactly."""
    attention, _ = _native()
    big, up, down = (500, 501, 499) if dtype == torch.float16 else (8, 9, 7)
    length = 65
    pages = (length + 15) // 16
    q = torch.full((1, 14, 64), big, dtype=dtype, device='cuda')
    q[:, 1::2].neg_()
    logical_k = torch.full((2, pages * 16, 64), big, dtype=dtype, device='cuda')
    logical_k[:, 0] = up
    logical_k[:, length - 1] = down
    k = logical_k.reshape(2, pages, 16, 64).permute(1, 0, 2, 3).contiguous()
    v = torch.randn(pages, 2, 16, 64, device='cuda').to(dtype)
    table = torch.arange(pages, device='cuda', dtype=torch.int32)[None]
    lens = torch.tensor([length], device='cuda', dtype=torch.int32)
    vflat = v.permute(1, 0, 2, 3).reshape(2, pages * 16, 64)
    for mode in MODES.values():
        out = attention.paged_decode_attention(q, k, v, table, lens, **mode)
        # even heads (q > 0) pick the largest key (token 0), odd heads the smallest (last token)
        for head in range(14):
            token = 0 if head % 2 == 0 else length - 1
            assert torch.equal(out[0, head], vflat[head // 7, token])


def test_online_state_is_not_rounded_per_page():
    """Mean of 32 ones and 4065 copies of 1 + 2^-10 is exactly 1 + 2^-10 in fp16
    (test/test_cuda_gqa_precision.py:69-79); rounding the running state to fp16
    per tile would lose the small updates."""
    attention, _ = _native()
    length = 4097
    pages = (length + 15) // 16
    q = torch.zeros(1, 14, 64, dtype=torch.float16, device='cuda')
    k = torch.zeros(pages, 2, 16, 64, dtype=torch.float16, device='cuda')
    v = torch.full((pages, 2, 16, 64), 1 + 2 ** -10, dtype=torch.float16, device='cuda')
    v[:2] = 1  # tokens 0..31
    table = torch.arange(pages, device='cuda', dtype=torch.int32)[None]
    lens = torch.tensor([length], device='cuda', dtype=torch.int32)
    for mode in MODES.values():
        for pps in (0, 4, 128):
            out = attention.paged_decode_attention(q, k, v, table, lens, **{'pages_per_split': pps, **mode})
            assert torch.equal(out, torch.full_like(out, 1 + 2 ** -10))


def test_fp32_large_values_stay_finite():
    """+-2e38 V with uniform weights: the normalised running state cannot overflow
    (test/test_cuda_paged_attention.py:102-112)."""
    attention, _ = _native()
    length = 65
    pages = (length + 3) // 4
    q = torch.zeros(1, 6, 33, device='cuda')
    k = torch.zeros(pages, 2, 4, 33, device='cuda')
    v = torch.empty(pages, 2, 4, 33, device='cuda')
    v[:, 0] = 2e38
    v[:, 1] = -2e38
    table = torch.arange(pages, device='cuda', dtype=torch.int64)[None]
    lens = torch.tensor([length], device='cuda', dtype=torch.int64)
    for pps in (0, 2):
        out = attention.paged_decode_attention(q, k, v, table, lens, pages_per_split=pps)
        assert torch.isfinite(out).all()
        expected = torch.empty_like(out)
        expected[0, :3] = 2e38
        expected[0, 3:] = -2e38
        torch.testing.assert_close(out, expected, rtol=5e-6, atol=0)


@pytest.mark.parametrize('heads,dim,dtype', [
    ((1, 1), 33, 'float32'), ((4, 4), 64, 'bfloat16'), ((14, 2), 64, 'float16'),
    ((14, 1), 64, 'bfloat16'), ((16, 1), 128, 'bfloat16'), ((24, 1), 128, 'bfloat16'),
    ((6, 2), 257, 'float16'), ((8, 8), 256, 'bfloat16'), ((32, 4), 256, 'float16'),
])
def test_head_ratios_and_dims(heads, dim, dtype):
    spec = dict(batch=3, q_heads=heads[0], kv_heads=heads[1], head_dim=dim, block_size=16,
                pool=('factor', 1.5), lens=('fixed', [1, 40, 250]), dtype=dtype,
                value_scale=1.0, seed=900 + dim + heads[0])
    inputs = make_inputs(spec)
    t, out = _append_and_decode(inputs)
    expected = _oracle(inputs, to_numpy(t['key_pool']), to_numpy(t['value_pool']))
    assert_attention_close(as_float(out), expected, dtype)


def test_fp64_per_head_restatement_agrees_on_fp32():
    """Cross-check against the reference tests' fp64 per-head loop (test_cuda_gqa.py:14-23)."""
    inputs = make_inputs('edge_bs3_d33_fp32')
    t, out = _append_and_decode(inputs)
    key_pool, value_pool = to_numpy(t['key_pool']), to_numpy(t['value_pool'])
    from oracle import gather_sequence
    bs = inputs['spec']['block_size']
    for b, length in enumerate(inputs['context_lens']):
        k = gather_sequence(key_pool, inputs['block_table'][b], int(length))
        v = gather_sequence(value_pool, inputs['block_table'][b], int(length))
        expected = decode_fp64_per_head(inputs['q'][b], k, v)
        np.testing.assert_allclose(as_float(out)[b], expected, rtol=2e-4, atol=2e-5)


def test_strided_and_broadcast_queries_and_out():
    attention, _ = _native()
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    q = t['q']
    base = attention.paged_decode_attention(q, t['key_pool'], t['value_pool'], t['block_table'],
                                            t['context_lens'])
    storage = torch.zeros(3, 60, 140, dtype=q.dtype, device='cuda')
    strided = storage[:, 1:57:2, 5:133]
    strided.copy_(q)
    out_storage = torch.zeros(3, 30, 150, dtype=q.dtype, device='cuda')
    out = out_storage[:, 1:29, 3:131]
    result = attention.paged_decode_attention(strided, t['key_pool'], t['value_pool'],
                                              t['block_table'], t['context_lens'], out=out)
    assert result.data_ptr() == out.data_ptr()
    assert torch.equal(out, base)
    assert (out_storage[:, 0] == 0).all() and (out_storage[:, :, :3] == 0).all()
    broadcast = q[:, :1].expand_as(q)
    assert broadcast.stride(1) == 0
    got = attention.paged_decode_attention(broadcast, t['key_pool'], t['value_pool'],
                                           t['block_table'], t['context_lens'])
    again = attention.paged_decode_attention(broadcast.contiguous(), t['key_pool'],
                                             t['value_pool'], t['block_table'], t['context_lens'])
    assert torch.equal(got, again)


def test_int64_tables_and_lengths_match_int32():
    attention, _ = _native()
    inputs = make_inputs('qwen72b_bf16_small')
    t = workload_tensors(inputs)
    a = attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], t['block_table'],
                                         t['context_lens'])
    b = attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'],
                                         t['block_table'].long(), t['context_lens'].long())
    assert torch.equal(a, b)


def test_inputs_unchanged_and_repeatable():
    attention, _ = _native()
    inputs = make_inputs('qwen3_8b_bf16_small')
    t = workload_tensors(inputs)
    before = {k: v.clone() for k, v in t.items()}
    first = attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'],
                                             t['block_table'], t['context_lens'])
    second = attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'],
                                              t['block_table'], t['context_lens'])
    assert torch.equal(first, second)
    assert first.data_ptr() != second.data_ptr()
    for key, tensor in t.items():
        assert torch.equal(tensor.view(torch.uint8) if tensor.dtype.is_floating_point else tensor,
                           before[key].view(torch.uint8) if tensor.dtype.is_floating_point else before[key])


def test_repeated_calls_are_bit_identical_on_every_default_path():
    """The same inputs give the same bits on every call: each split walks its
    pages in a fixed order and the merge sums the splits in a fixed order, on
    a multi-wave grid (first-split schedule), the one-call step, contiguous
    caches and chunk query tiles alike."""
    attention, cache = _native()
    spec = dict(batch=128, q_heads=28, kv_heads=4, head_dim=128, block_size=16, pool=('factor', 1.25),
                lens=('uniform', 100, 700), dtype='bfloat16', value_scale=0.5, seed=777)
    inputs = make_inputs(spec)
    t = workload_tensors(inputs)

    def same(fn):
        first = fn().clone()
        for _ in range(3):
            again = fn()
            torch.cuda.synchronize()
            assert torch.equal(first.view(torch.int16), again.view(torch.int16))

    same(lambda: attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], t['block_table'],
                                                  t['context_lens']))
    same(lambda: attention.paged_decode_with_append(t['q'], t['key_new'], t['value_new'], t['key_pool'],
                                                    t['value_pool'], t['block_table'], t['context_lens']))
    gen = torch.Generator(device='cuda').manual_seed(5)
    kc = torch.randn((64, 4, 512, 128), generator=gen, device='cuda').to(torch.bfloat16)
    vc = torch.randn((64, 4, 512, 128), generator=gen, device='cuda').to(torch.bfloat16)
    qc = torch.randn((64, 28, 128), generator=gen, device='cuda').to(torch.bfloat16)
    lc = torch.randint(1, 513, (64,), generator=torch.Generator().manual_seed(6)).to(torch.int32).cuda()
    same(lambda: attention.contiguous_decode_attention(qc, kc, vc, lc))
    qt = torch.randn((8, 28, 32, 128), generator=gen, device='cuda').to(torch.bfloat16)
    lens = t['context_lens'][:8].clamp(min=32)
    same(lambda: attention.paged_chunk_attention(qt, t['key_pool'], t['value_pool'], t['block_table'][:8], lens))


@pytest.mark.parametrize('pps', [32, 4, 2, 1])
def test_merge_paths_for_many_splits(pps):
    """Rows of up to 8 pieces (warp per row), 64 and 128 pieces (a CTA per row whose
    warps share the pieces) and 256 (a CTA per row looping over them): the
    same output within the parity bar, and a corrupted page in one split
    poisons exactly its sequence."""
    attention, _ = _native()
    lens = [4096, 1000, 16, 2100, 1]
    spec = dict(batch=len(lens), q_heads=28, kv_heads=4, head_dim=128, block_size=16,
                pool=('factor', 1.2), lens=('fixed', lens), dtype='bfloat16', value_scale=0.5, seed=808 + pps)
    inputs = make_inputs(spec)
    t, out = _append_and_decode(inputs, pages_per_split=pps)
    assert attention.paged_decode_plan(28, t['key_pool'], 4096, batch=len(lens), pages_per_split=pps)[2] == \
        -(-256 // pps)
    expected = _oracle(inputs, to_numpy(t['key_pool']), to_numpy(t['value_pool']))
    assert_attention_close(as_float(out), expected, 'bfloat16')
    table = t['block_table'].clone()
    table[0, 200] = t['key_pool'].shape[0]          # a page in a middle split of the longest sequence
    bad = attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], table, t['context_lens'],
                                           pages_per_split=pps)
    torch.cuda.synchronize()
    values = as_float(bad)
    assert np.isnan(values[0]).all() and np.isfinite(values[1:]).all()
    from micro_vllm_b200 import _native as native
    native.check(native.library().mv_clear_device_status(torch.cuda.current_device()))
