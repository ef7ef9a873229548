"""GPU parity of the one-call decode step (append + attend, ``mv_paged_decode_append``).

Where the split-grid tensor-core kernel runs, the CTA attending a sequence's
last page writes the step's new K/V row itself; every other plan runs the
append kernel first. Either way the pools must be bit-identical to the
reference's own append (the golden digests) and to the two-call path, and the
output bit-identical to the two-call path and within the parity bar of the
oracle.
"""
import numpy as np
import pytest
import torch

from oracle import decode_float
from tests.golden.cases import array_digest, make_inputs
from tests.golden.make_golden import GOLDEN_CASES
from tests.helpers import as_float, assert_attention_close, to_numpy, workload_tensors

pytestmark = pytest.mark.gpu

MODES = {
    'auto': {},                               # split grid: append fused into the decode kernel
    'fused_merge': dict(fused_merge=True),    # split grid, last split CTA merges: append fused
    'split4': dict(pages_per_split=4),        # split grid, many splits: append fused
    'wide': dict(wide=True),                  # split grid, wide shape: append fused
    'persistent': dict(persistent=True),      # append kernel first, then the persistent kernel
    'cluster': dict(cluster=True),            # append kernel first, then the cluster kernel
    'simt': dict(force_simt=True),            # CUDA-core kernel: append fused (element-wise)
    'cuda_core_math': dict(cuda_core_math=True),  # split grid, fp32 FMA math: append fused
}


def _ops():
    from micro_vllm_b200 import cuda_attention, cuda_paged_cache
    return cuda_attention, cuda_paged_cache


def _two_calls(t, table=None, lens=None, key=None, value=None, **mode):
    attention, cache = _ops()
    table = t['block_table'] if table is None else table
    lens = t['context_lens'] if lens is None else lens
    key_pool, value_pool = t['key_pool'].clone(), t['value_pool'].clone()
    cache.write_paged_kv(t['key_new'] if key is None else key, t['value_new'] if value is None else value,
                         key_pool, value_pool, table, positions=lens, positions_are_end=True)
    out = attention.paged_decode_attention(t['q'], key_pool, value_pool, table, lens, **mode)
    torch.cuda.synchronize()
    return key_pool, value_pool, out


def _one_call(t, table=None, lens=None, key=None, value=None, **mode):
    attention, _ = _ops()
    table = t['block_table'] if table is None else table
    lens = t['context_lens'] if lens is None else lens
    key_pool, value_pool = t['key_pool'].clone(), t['value_pool'].clone()
    out = attention.paged_decode_with_append(
        t['q'], t['key_new'] if key is None else key, t['value_new'] if value is None else value,
        key_pool, value_pool, table, lens, **mode)
    torch.cuda.synchronize()
    return key_pool, value_pool, out


def _same_bits(a, b):
    return torch.equal(a.view(torch.int16) if a.element_size() == 2 else a.view(torch.int32),
                       b.view(torch.int16) if b.element_size() == 2 else b.view(torch.int32))


@pytest.mark.parametrize('name', GOLDEN_CASES)
@pytest.mark.parametrize('mode', list(MODES))
def test_one_call_step_matches_golden_pools_two_calls_and_the_oracle(name, mode):
    from pathlib import Path
    inputs = make_inputs(name)
    dtype = inputs['spec']['dtype']
    t = workload_tensors(inputs)
    key_pool, value_pool, out = _one_call(t, **MODES[mode])
    with np.load(Path(__file__).resolve().parent / 'golden' / f'{name}.npz') as fixture:
        assert array_digest(to_numpy(key_pool)) == str(fixture['key_pool_digest'])
        assert array_digest(to_numpy(value_pool)) == str(fixture['value_pool_digest'])
    ref_k, ref_v, ref_out = _two_calls(t, **MODES[mode])
    assert _same_bits(key_pool, ref_k) and _same_bits(value_pool, ref_v)
    assert _same_bits(out, ref_out)
    expected = decode_float(inputs['q'], to_numpy(key_pool), to_numpy(value_pool), inputs['block_table'],
                            inputs['context_lens'], inputs['q'].shape[-1] ** -0.5, dtype)
    assert_attention_close(as_float(out), expected, dtype)


@pytest.mark.parametrize('name', ['qwen7b_bf16_small', 'qwen05b_fp16', 'edge_bs64_d64_bf16'])
def test_every_slot_of_the_last_page(name):
    """Lengths that put the new token in each of the 16 slots, and page starts/ends."""
    inputs = make_inputs(name)
    t = workload_tensors(inputs)
    bs = t['key_pool'].shape[2]
    capacity = t['block_table'].shape[1] * bs
    for base in (0, bs, capacity - bs):
        for slot in range(0, bs, max(1, bs // 16)):
            lens = torch.full_like(t['context_lens'], base + slot + 1)
            lens[0] = min(capacity, max(1, base + slot + 1 - 3))
            for mode in (MODES['auto'], MODES['split4']):
                k1, v1, o1 = _one_call(t, lens=lens, **mode)
                k2, v2, o2 = _two_calls(t, lens=lens, **mode)
                assert _same_bits(k1, k2) and _same_bits(v1, v2)
                assert _same_bits(o1, o2)


def test_lengths_outside_the_plan_still_append_like_the_append_kernel():
    """Length 0 (no write), above max_context_len (NaN output, row still written),
    beyond the table (no write), negative (no write)."""
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    capacity = t['block_table'].shape[1] * 16
    lens = t['context_lens'].clone()
    lens[0] = 0
    lens[1] = capacity + 1
    lens[2] = -5
    bound = int(inputs['context_lens'].max())
    for mode in MODES.values():
        k1, v1, o1 = _one_call(t, lens=lens, **mode)
        k2, v2, o2 = _two_calls(t, lens=lens, **mode)
        assert _same_bits(k1, k2) and _same_bits(v1, v2)
        out = as_float(o1)
        assert (out[0] == 0).all() and np.isnan(out[1]).all() and np.isnan(out[2]).all()
    attention, _ = _ops()
    lens = t['context_lens'].clone()
    lens[1] = bound + 20  # inside the table, above the bound the caller promised
    for mode in (MODES['auto'], MODES['simt']):
        key_pool, value_pool = t['key_pool'].clone(), t['value_pool'].clone()
        out = attention.paged_decode_with_append(t['q'], t['key_new'], t['value_new'], key_pool, value_pool,
                                                 t['block_table'], lens, max_context_len=bound, **mode)
        k2, v2, _ = _two_calls(t, lens=lens, max_context_len=bound, **mode)
        torch.cuda.synchronize()
        assert _same_bits(key_pool, k2) and _same_bits(value_pool, v2)
        assert np.isnan(as_float(out)[1]).all()


def test_corrupted_page_ids_skip_the_write_and_poison_only_that_sequence():
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    lens = inputs['context_lens']
    victim = int(np.argmax(lens))
    last = -(-int(lens[victim]) // 16) - 1
    for page in (last, 0):
        for bad in (-1, t['key_pool'].shape[0]):
            table = t['block_table'].clone()
            table[victim, page] = bad
            for mode in MODES.values():
                k1, v1, o1 = _one_call(t, table=table, **mode)
                k2, v2, o2 = _two_calls(t, table=table, **mode)
                assert _same_bits(k1, k2) and _same_bits(v1, v2)
                values = as_float(o1)
                assert np.isnan(values[victim]).all()
                assert np.isfinite(np.delete(values, victim, axis=0)).all()


def test_rows_sliced_from_a_fused_projection_and_unaligned_rows():
    """New K/V as views of one [B, Hq + 2 Hkv, D] projection output (16-byte aligned:
    fused in the kernel) and as views offset by one element (not aligned: the
    append kernel runs first); both must equal the two-call step."""
    inputs = make_inputs('qwen72b_bf16_small')
    t = workload_tensors(inputs)
    batch, hkv, _, dim = t['key_new'].shape
    hq = t['q'].shape[1]
    for offset in (0, 1):
        qkv = torch.randn(batch, hq + 2 * hkv, dim + offset, device='cuda').to(t['q'].dtype)
        key = qkv[:, hq:hq + hkv, offset:]
        value = qkv[:, hq + hkv:, offset:]
        k1, v1, o1 = _one_call(t, key=key, value=value)
        k2, v2, o2 = _two_calls(t, key=key.unsqueeze(2), value=value.unsqueeze(2))
        assert _same_bits(k1, k2) and _same_bits(v1, v2)
        assert _same_bits(o1, o2)


def test_int64_tables_and_lengths():
    inputs = make_inputs('qwen3_8b_bf16_small')
    t = workload_tensors(inputs)
    table64 = t['block_table'].to(torch.int64)
    lens64 = t['context_lens'].to(torch.int64)
    k1, v1, o1 = _one_call(t, table=table64, lens=lens64)
    k2, v2, o2 = _two_calls(t)
    assert _same_bits(k1, k2) and _same_bits(v1, v2) and _same_bits(o1, o2)


def test_one_call_step_in_a_cuda_graph_replays_steps():
    """Capture the step once; each replay appends at the current lengths."""
    attention, _ = _ops()
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    lens = (t['context_lens'] - 2).clone()
    key_pool, value_pool = t['key_pool'].clone(), t['value_pool'].clone()
    out = torch.empty_like(t['q'])
    bound = t['block_table'].shape[1] * 16
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        attention.paged_decode_with_append(t['q'], t['key_new'], t['value_new'], key_pool, value_pool,
                                           t['block_table'], lens, max_context_len=bound, out=out)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        attention.paged_decode_with_append(t['q'], t['key_new'], t['value_new'], key_pool, value_pool,
                                           t['block_table'], lens, max_context_len=bound, out=out)
    for _ in range(2):
        lens += 1
        graph.replay()
    torch.cuda.synchronize()
    ref = dict(t)
    ref['key_pool'], ref['value_pool'] = t['key_pool'].clone(), t['value_pool'].clone()
    _, cache = _ops()
    for step in (-2, -1, 0):
        cache.write_paged_kv(t['key_new'], t['value_new'], ref['key_pool'], ref['value_pool'],
                             t['block_table'], positions=t['context_lens'] + step, positions_are_end=True)
    expected = attention.paged_decode_attention(t['q'], ref['key_pool'], ref['value_pool'], t['block_table'],
                                                t['context_lens'], max_context_len=bound)
    torch.cuda.synchronize()
    assert _same_bits(key_pool, ref['key_pool']) and _same_bits(value_pool, ref['value_pool'])
    assert _same_bits(out, expected)


@pytest.mark.parametrize('mode', ['auto', 'split4', 'persistent', 'simt'])
def test_bound_step_matches_the_one_off_calls(mode):
    attention, _ = _ops()
    inputs = make_inputs('qwen72b_bf16_small')
    t = workload_tensors(inputs)
    pools = (t['key_pool'].clone(), t['value_pool'].clone())
    step = attention.PagedDecodeStep(*pools, t['block_table'], num_q_heads=t['q'].shape[1], **MODES[mode])
    out = step(t['q'], t['context_lens'], key=t['key_new'], value=t['value_new'])
    k2, v2, o2 = _one_call(t, **MODES[mode])
    assert _same_bits(pools[0], k2) and _same_bits(pools[1], v2) and _same_bits(out, o2)
    # Attention only, 4-D query, int64 lengths, caller-provided output.
    q4 = t['q'].unsqueeze(2)
    out2 = torch.empty_like(t['q'])
    step(q4, t['context_lens'].to(torch.int64), out2)
    expected = attention.paged_decode_attention(t['q'], *pools, t['block_table'], t['context_lens'],
                                                **MODES[mode])
    torch.cuda.synchronize()
    assert _same_bits(out2, expected)
    assert step.plan == attention.paged_decode_plan(t['q'].shape[1], pools[0], t['block_table'].shape[1] * 16,
                                                    batch=t['q'].shape[0], **{k: v for k, v in MODES[mode].items()
                                                                              if k != 'fused_merge'})


def test_bound_step_rejects_changed_shapes_and_aliases():
    attention, _ = _ops()
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    step = attention.PagedDecodeStep(t['key_pool'], t['value_pool'], t['block_table'], num_q_heads=28)
    with pytest.raises(RuntimeError, match='bound shape'):
        step(t['q'][:, :14], t['context_lens'])
    with pytest.raises(RuntimeError, match='bound shape'):
        step(t['q'].float(), t['context_lens'])
    with pytest.raises(RuntimeError, match='context lengths'):
        step(t['q'], t['context_lens'][:1])
    with pytest.raises(RuntimeError, match='both new K and V'):
        step(t['q'], t['context_lens'], key=t['key_new'])
    with pytest.raises(RuntimeError, match='alias'):
        alias = t['key_pool'][:t['q'].shape[0], :, 0, :]
        step(t['q'], t['context_lens'], key=alias, value=t['value_new'])
    with pytest.raises(RuntimeError, match='out must be'):
        step(t['q'], t['context_lens'], torch.empty(1, 28, 128, dtype=t['q'].dtype, device='cuda'))


@pytest.mark.parametrize('lens', [('uniform', 100, 700), ('uniform', 1, 700),
                                  ('fixed', [700] * 120 + [0, 1, 15, 16, 17, 511, 512, 513])])
def test_first_split_schedule_of_multi_wave_grids(lens):
    """Grids of more than one wave of CTAs take a first split twice the split
    size, a second of the split size and later ones of a quarter of it (at
    least 16 pages; while that keeps the plan at 8 splits or fewer),
    dispatched split-major. Check the shape the plan reports, then the
    one-call step and the two-call path against each other, the uniform-split
    plan of the same size, and the oracle, with empty and page-edge lengths."""
    spec = dict(batch=128, q_heads=28, kv_heads=4, head_dim=128, block_size=16, pool=('factor', 1.25),
                lens=lens, dtype='bfloat16', value_scale=0.5, seed=4242)
    inputs = make_inputs(spec)
    t = workload_tensors(inputs)
    attention, _ = _ops()
    max_pages = t['block_table'].shape[1]
    path, pps, splits = attention.paged_decode_plan(28, t['key_pool'], max_pages * 16, batch=128)
    assert path == 'tma_mma' and 2 * pps < max_pages
    later = max(16, pps // 4)
    graded = 1 if max_pages <= 2 * pps else 2 if max_pages <= 3 * pps else 2 + -(-(max_pages - 3 * pps) // later)
    if graded > 8:
        later = pps
    expected = 1 if max_pages <= 2 * pps else 2 if max_pages <= 3 * pps else 2 + -(-(max_pages - 3 * pps) // later)
    assert splits == expected   # splits of 2 x pps, pps, then `later` pages (graded up to 8 splits)
    key_pool, value_pool, out = _one_call(t)
    ref_k, ref_v, ref_out = _two_calls(t)
    assert _same_bits(key_pool, ref_k) and _same_bits(value_pool, ref_v)
    assert _same_bits(out, ref_out)
    _, _, uniform = _two_calls(t, pages_per_split=pps)
    expected = decode_float(inputs['q'], to_numpy(key_pool), to_numpy(value_pool), inputs['block_table'],
                            inputs['context_lens'], 128 ** -0.5, 'bfloat16')
    assert_attention_close(as_float(out), expected, 'bfloat16')
    assert_attention_close(as_float(uniform), expected, 'bfloat16')
    empty = inputs['context_lens'] == 0
    assert (as_float(out)[empty] == 0).all()


def test_bound_step_repeats_with_the_same_tensors_skip_the_checks_and_stay_exact():
    """A repeat of the last call (same tensor objects and storage, same stream)
    goes straight to the packed C call; it must see in-place changes to the
    inputs, match the one-off call bit for bit, and fall back to the checked
    path when any tensor changes."""
    attention, _ = _ops()
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    pools = (t['key_pool'].clone(), t['value_pool'].clone())
    step = attention.PagedDecodeStep(*pools, t['block_table'], num_q_heads=t['q'].shape[1])
    q, lens = t['q'].clone(), t['context_lens'].clone()
    key, value = t['key_new'][:, :, 0].clone(), t['value_new'][:, :, 0].clone()
    out = torch.empty_like(q)
    step(q, lens, out, key=key, value=value)
    assert len(step._fast) == 1
    for scale in (0.5, -2.0):
        q.mul_(scale)                              # same storage, new values
        key.mul_(scale)
        step(q, lens, out, key=key, value=value)  # the repeat
        ref_pools = (t['key_pool'].clone(), t['value_pool'].clone())
        expected = attention.paged_decode_with_append(q, key, value, *ref_pools, t['block_table'], lens)
        torch.cuda.synchronize()
        assert _same_bits(out, expected)
        assert _same_bits(pools[0], ref_pools[0]) and _same_bits(pools[1], ref_pools[1])
    other = torch.empty_like(q)
    step(q, lens, other, key=key, value=value)    # a different output tensor: checked again
    torch.cuda.synchronize()
    assert _same_bits(other, out)
    assert len(step._fast) == 2
    with pytest.raises(RuntimeError, match='bound shape'):
        step(q[:1], lens, out, key=key, value=value)
