"""GPU parity of the per-warp stream schedule (``paged_decode_stream_kernel``).

The schedule runs on request (``schedule='stream'``; measured slower than the
split grid, so the library never picks it by itself). It is checked at full
size on the benchmark workloads (``test_stream_full_size_matches_the_oracle``)
and here, forced on small cases with items from one
page up, so the queue holds many items of every size and each warp's TMA ring
crosses item boundaries, and every edge the split grid covers is checked on
this schedule too: the fused append (bit-exact against the reference's own
append and against the two-call step), RoPE, corrupted page IDs, empty and
out-of-range lengths, int64 tables, CUDA-graph replay and repeated calls
(bit-identical: the item a warp takes never changes the result).
"""
import numpy as np
import pytest
import torch

from oracle import append_tokens, decode_float
from oracle.rope import apply_rope as oracle_rope
from tests.golden.cases import array_digest, make_inputs
from tests.helpers import as_float, assert_attention_close, to_numpy, workload_tensors

pytestmark = pytest.mark.gpu

# Golden cases with the stream schedule's shape (bf16/fp16, page 16, head_dim 64/128, group <= 8).
STREAM_CASES = ['qwen7b_bf16_small', 'qwen3_8b_bf16_small', 'qwen72b_bf16_small', 'qwen05b_bf16',
                'qwen05b_fp16']
ITEM_PAGES = [0, 1, 3, 8, 64]     # 0: the library's choice


def _ops():
    from micro_vllm_b200 import cuda_attention, cuda_paged_cache
    return cuda_attention, cuda_paged_cache


def _bits(t):
    return t.view(torch.int16) if t.element_size() == 2 else t.view(torch.int32)


def _same_bits(a, b):
    return torch.equal(_bits(a), _bits(b))


def _one_call(t, table=None, lens=None, **mode):
    attention, _ = _ops()
    table = t['block_table'] if table is None else table
    lens = t['context_lens'] if lens is None else lens
    key_pool, value_pool = t['key_pool'].clone(), t['value_pool'].clone()
    out = attention.paged_decode_with_append(t['q'], t['key_new'], t['value_new'], key_pool, value_pool,
                                             table, lens, **mode)
    torch.cuda.synchronize()
    return key_pool, value_pool, out


def _two_calls(t, table=None, lens=None, **mode):
    attention, cache = _ops()
    table = t['block_table'] if table is None else table
    lens = t['context_lens'] if lens is None else lens
    key_pool, value_pool = t['key_pool'].clone(), t['value_pool'].clone()
    cache.write_paged_kv(t['key_new'], t['value_new'], key_pool, value_pool, table, positions=lens,
                         positions_are_end=True)
    out = attention.paged_decode_attention(t['q'], key_pool, value_pool, table, lens, **mode)
    torch.cuda.synchronize()
    return key_pool, value_pool, out


def _oracle(inputs, key_pool, value_pool):
    return decode_float(inputs['q'], to_numpy(key_pool), to_numpy(value_pool), inputs['block_table'],
                        inputs['context_lens'], inputs['q'].shape[-1] ** -0.5, inputs['spec']['dtype'])


def test_plan_reports_the_stream_schedule():
    attention, _ = _ops()
    t = workload_tensors(make_inputs('qwen7b_bf16_small'))
    for pps in (1, 3, 8, 64):
        assert attention.paged_decode_plan(28, t['key_pool'], 4096, batch=3, pages_per_split=pps,
                                           schedule='stream') == ('tma_mma_stream', pps, -(-256 // pps))
    # Never picked by itself; 'split' is the default.
    assert attention.paged_decode_plan(28, t['key_pool'], 4096, batch=3)[0] == 'tma_mma'
    assert attention.paged_decode_plan(28, t['key_pool'], 4096, batch=64)[0] == 'tma_mma'
    assert attention.paged_decode_plan(28, t['key_pool'], 4096, batch=64, schedule='split')[0] == 'tma_mma'
    assert attention.paged_decode_plan(28, t['key_pool'], 4096, batch=64, schedule='stream') == \
        ('tma_mma_stream', 8, 32)
    # Shapes it does not take: an error when forced.
    with pytest.raises(RuntimeError, match='MV_FLAG_STREAM'):
        attention.paged_decode_plan(28, t['key_pool'].float(), 4096, batch=3, schedule='stream')
    with pytest.raises(RuntimeError, match='MV_FLAG_STREAM'):
        attention.paged_decode_plan(28, t['key_pool'], 4096, batch=3, pages_per_split=65, schedule='stream')


@pytest.mark.parametrize('name', STREAM_CASES)
@pytest.mark.parametrize('pps', ITEM_PAGES)
def test_stream_step_matches_golden_pools_two_calls_and_the_oracle(name, pps):
    from pathlib import Path
    inputs = make_inputs(name)
    t = workload_tensors(inputs)
    mode = dict(schedule='stream', pages_per_split=pps)
    key_pool, value_pool, out = _one_call(t, **mode)
    with np.load(Path(__file__).resolve().parent / 'golden' / f'{name}.npz') as fixture:
        assert array_digest(to_numpy(key_pool)) == str(fixture['key_pool_digest'])
        assert array_digest(to_numpy(value_pool)) == str(fixture['value_pool_digest'])
    k2, v2, o2 = _two_calls(t, **mode)
    assert _same_bits(key_pool, k2) and _same_bits(value_pool, v2) and _same_bits(out, o2)
    assert_attention_close(as_float(out), _oracle(inputs, key_pool, value_pool), inputs['spec']['dtype'])


@pytest.mark.parametrize('lens', [[1], [16], [17], [1, 1, 1], [4096, 1, 33], [5000, 40, 7, 3000],
                                  [16] * 37, [1029, 700, 1] * 5, list(range(1, 1200, 19))])
@pytest.mark.parametrize('pps', [1, 2, 5, 16])
def test_stream_length_mixes(lens, pps):
    """Items of every size from one page: full items, ragged last items sorted
    by size, single-item sequences (final output) and split ones (merge)."""
    spec = dict(batch=len(lens), q_heads=28, kv_heads=4, head_dim=128, block_size=16,
                pool=('factor', 1.3), lens=('fixed', lens), dtype='bfloat16', value_scale=0.5,
                seed=71 + len(lens) + pps)
    inputs = make_inputs(spec)
    t = workload_tensors(inputs)
    key_pool, value_pool, out = _one_call(t, schedule='stream', pages_per_split=pps)
    assert_attention_close(as_float(out), _oracle(inputs, key_pool, value_pool), 'bfloat16')
    _, _, split_out = _one_call(t, schedule='split')
    assert_attention_close(as_float(out), as_float(split_out), 'bfloat16')


@pytest.mark.parametrize('pps', [3, 8])
def test_many_sequences_share_item_sizes(pps):
    """500 sequences whose ragged last items share sizes many times over, and
    some not attended: every CTA of the grid must number the items the same
    way, or some items run twice and others never (the append of a skipped
    last item would be missing)."""
    lens = [1 + (b * 37) % 400 for b in range(500)]
    lens[7] = lens[123] = 0
    spec = dict(batch=len(lens), q_heads=28, kv_heads=4, head_dim=128, block_size=16,
                pool=('factor', 1.1), lens=('fixed', lens), dtype='bfloat16', value_scale=0.5, seed=515 + pps)
    inputs = make_inputs(spec)
    t = workload_tensors(inputs)
    mode = dict(schedule='stream', pages_per_split=pps)
    key_pool, value_pool, out = _one_call(t, **mode)
    k2, v2, o2 = _two_calls(t, **mode)
    assert _same_bits(key_pool, k2) and _same_bits(value_pool, v2) and _same_bits(out, o2)
    assert_attention_close(as_float(out), _oracle(inputs, key_pool, value_pool), 'bfloat16')


def test_unattended_and_out_of_range_lengths_append_like_the_append_kernel():
    """Length 0 (zeros, no write), above the table (NaN, no write), negative
    (NaN, no write), above the caller's bound (NaN, row still written)."""
    attention, _ = _ops()
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    capacity = t['block_table'].shape[1] * 16
    lens = t['context_lens'].clone()
    lens[0] = 0
    lens[1] = capacity + 1
    lens[2] = -5
    for pps in (1, 8):
        mode = dict(schedule='stream', pages_per_split=pps)
        k1, v1, o1 = _one_call(t, lens=lens, **mode)
        k2, v2, _ = _two_calls(t, lens=lens, **mode)
        assert _same_bits(k1, k2) and _same_bits(v1, v2)
        out = as_float(o1)
        assert (out[0] == 0).all() and np.isnan(out[1]).all() and np.isnan(out[2]).all()
    bound = int(inputs['context_lens'].max())
    lens = t['context_lens'].clone()
    lens[1] = bound + 20
    key_pool, value_pool = t['key_pool'].clone(), t['value_pool'].clone()
    out = attention.paged_decode_with_append(t['q'], t['key_new'], t['value_new'], key_pool, value_pool,
                                             t['block_table'], lens, max_context_len=bound, schedule='stream',
                                             pages_per_split=2)
    k2, v2, _ = _two_calls(t, lens=lens, max_context_len=bound, schedule='stream', pages_per_split=2)
    torch.cuda.synchronize()
    assert _same_bits(key_pool, k2) and _same_bits(value_pool, v2)
    values = as_float(out)
    assert np.isnan(values[1]).all() and np.isfinite(values[[0, 2]]).all()


@pytest.mark.parametrize('where', ['last', 'first', 'middle'])
def test_corrupted_page_id_poisons_that_sequence_and_raises_the_status(where):
    """A page ID outside the pool: NaN for that sequence, the status bit, no read
    of the page; the new row is still written when its own page ID is valid,
    exactly as the append kernel writes it."""
    from micro_vllm_b200 import _native
    lib = _native.library()
    device = torch.cuda.current_device()
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    lens = inputs['context_lens']
    victim = int(np.argmax(lens))
    pages = -(-int(lens[victim]) // 16)
    page = {'last': pages - 1, 'first': 0, 'middle': pages // 2}[where]
    for bad in (-1, t['key_pool'].shape[0]):
        table = t['block_table'].clone()
        table[victim, page] = bad
        for pps in (1, 4, 64):
            _native.check(lib.mv_clear_device_status(device))
            mode = dict(schedule='stream', pages_per_split=pps)
            k1, v1, o1 = _one_call(t, table=table, **mode)
            status = ctypes_status(lib, device)
            k2, v2, _ = _two_calls(t, table=table, **mode)
            assert _same_bits(k1, k2) and _same_bits(v1, v2)
            values = as_float(o1)
            assert np.isnan(values[victim]).all()
            assert np.isfinite(np.delete(values, victim, axis=0)).all()
            assert status & _native.DEVICE_STATUS_BAD_PAGE_ID
    _native.check(lib.mv_clear_device_status(device))


def ctypes_status(lib, device):
    import ctypes
    from micro_vllm_b200 import _native
    value = ctypes.c_uint32(0)
    _native.check(lib.mv_device_status(device, ctypes.byref(value)))
    return value.value


@pytest.mark.parametrize('name', ['qwen7b_bf16_small', 'qwen72b_bf16_small', 'qwen05b_fp16'])
@pytest.mark.parametrize('pps', [0, 2])
def test_fused_rope_equals_rotate_then_step_and_the_oracle(name, pps):
    attention, _ = _ops()
    from micro_vllm_b200.rope import apply_rope, rope_tables
    inputs = make_inputs(name)
    dtype = inputs['spec']['dtype']
    t = workload_tensors(inputs)
    dim = t['q'].shape[-1]
    cap = t['block_table'].shape[1] * t['key_pool'].shape[2]
    cos, sin = rope_tables(cap, dim, 1e6, dtype=t['q'].dtype, device=t['q'].device)
    key, value = t['key_new'][:, :, 0], t['value_new'][:, :, 0]
    mode = dict(schedule='stream', pages_per_split=pps)
    pools = (t['key_pool'].clone(), t['value_pool'].clone())
    out = attention.paged_decode_with_append(t['q'], key, value, *pools, t['block_table'], t['context_lens'],
                                             rope=(cos, sin), **mode)
    q_rot = apply_rope(t['q'], cos, sin, positions=t['context_lens'], positions_are_end=True)
    k_rot = apply_rope(key, cos, sin, positions=t['context_lens'], positions_are_end=True)
    ref_pools = (t['key_pool'].clone(), t['value_pool'].clone())
    ref = attention.paged_decode_with_append(q_rot, k_rot, value, *ref_pools, t['block_table'],
                                             t['context_lens'], **mode)
    torch.cuda.synchronize()
    assert _same_bits(pools[0], ref_pools[0]) and _same_bits(pools[1], ref_pools[1])
    assert _same_bits(out, ref)
    lens = inputs['context_lens'].astype(np.int64)
    cos_np, sin_np = to_numpy(cos), to_numpy(sin)
    q_np = oracle_rope(inputs['q'], cos_np[lens - 1][:, None], sin_np[lens - 1][:, None], dtype)
    k_np = oracle_rope(inputs['key_new'][:, :, 0], cos_np[lens - 1][:, None], sin_np[lens - 1][:, None], dtype)
    kp, vp = inputs['key_pool'].copy(), inputs['value_pool'].copy()
    append_tokens(kp, vp, k_np[:, :, None], inputs['value_new'], inputs['block_table'], lens - 1)
    assert np.array_equal(to_numpy(pools[0]).view(np.uint8), kp.view(np.uint8))
    expected = decode_float(q_np, kp, vp, inputs['block_table'], inputs['context_lens'], dim ** -0.5, dtype)
    assert_attention_close(as_float(out), expected, dtype)


def test_int64_tables_and_lengths():
    inputs = make_inputs('qwen3_8b_bf16_small')
    t = workload_tensors(inputs)
    mode = dict(schedule='stream', pages_per_split=3)
    k1, v1, o1 = _one_call(t, table=t['block_table'].to(torch.int64), lens=t['context_lens'].to(torch.int64),
                           **mode)
    k2, v2, o2 = _one_call(t, **mode)
    assert _same_bits(k1, k2) and _same_bits(v1, v2) and _same_bits(o1, o2)


def test_repeated_calls_are_bit_identical_and_the_queue_resets():
    """The item queue's counters return to zero after every launch, whatever
    schedule shares the workspace in between; results never change."""
    attention, _ = _ops()
    cases = [workload_tensors(make_inputs(name)) for name in ('qwen7b_bf16_small', 'qwen72b_bf16_small')]
    first = None
    for _ in range(3):
        outs = []
        for t in cases:
            for mode in (dict(schedule='stream', pages_per_split=1), dict(schedule='split'),
                         dict(schedule='stream', pages_per_split=4), dict(fused_merge=True, pages_per_split=2)):
                outs.append(attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'],
                                                             t['block_table'], t['context_lens'], **mode))
        torch.cuda.synchronize()
        if first is None:
            first = outs
        else:
            assert all(_same_bits(a, b) for a, b in zip(first, outs))


def test_stream_step_in_a_cuda_graph_replays_steps():
    """Capture the one-call step once; each replay appends at the current lengths."""
    attention, cache = _ops()
    inputs = make_inputs('qwen72b_bf16_small')
    t = workload_tensors(inputs)
    lens = (t['context_lens'] - 2).clone()
    key_pool, value_pool = t['key_pool'].clone(), t['value_pool'].clone()
    out = torch.empty_like(t['q'])
    bound = t['block_table'].shape[1] * 16
    mode = dict(max_context_len=bound, schedule='stream', pages_per_split=2)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        attention.paged_decode_with_append(t['q'], t['key_new'], t['value_new'], key_pool, value_pool,
                                           t['block_table'], lens, out=out, **mode)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        attention.paged_decode_with_append(t['q'], t['key_new'], t['value_new'], key_pool, value_pool,
                                           t['block_table'], lens, out=out, **mode)
    for _ in range(2):
        lens += 1
        graph.replay()
    torch.cuda.synchronize()
    ref_k, ref_v = t['key_pool'].clone(), t['value_pool'].clone()
    for step in (-2, -1, 0):
        cache.write_paged_kv(t['key_new'], t['value_new'], ref_k, ref_v, t['block_table'],
                             positions=t['context_lens'] + step, positions_are_end=True)
    expected = attention.paged_decode_attention(t['q'], ref_k, ref_v, t['block_table'], t['context_lens'], **mode)
    torch.cuda.synchronize()
    assert _same_bits(key_pool, ref_k) and _same_bits(value_pool, ref_v)
    assert _same_bits(out, expected)


def test_bound_step_takes_the_stream_schedule():
    attention, _ = _ops()
    t = workload_tensors(make_inputs('qwen72b_bf16_small'))
    pools = (t['key_pool'].clone(), t['value_pool'].clone())
    step = attention.PagedDecodeStep(*pools, t['block_table'], num_q_heads=t['q'].shape[1], schedule='stream',
                                     pages_per_split=2)
    assert step.plan[0] == 'tma_mma_stream'
    out = step(t['q'], t['context_lens'], key=t['key_new'], value=t['value_new'])
    k2, v2, o2 = _one_call(t, schedule='stream', pages_per_split=2)
    assert _same_bits(pools[0], k2) and _same_bits(pools[1], v2) and _same_bits(out, o2)


@pytest.mark.slow
@pytest.mark.parametrize('name', ['qwen7b_bf16', 'qwen72b_bf16'])
def test_stream_full_size_matches_the_oracle(name):
    """The benchmark workloads at full size on the stream schedule: the append
    bit-exact, every sequence (Qwen2.5-7B) or 24 of 256 (Qwen2.5-72B) against
    the oracle."""
    from tests.test_gpu_full_size import _check_append, _check_attention, _extremes_and_stride
    from tests.golden.workloads import WORKLOADS, make_workload
    attention, _ = _ops()
    spec = WORKLOADS[name]
    data = make_workload(spec, spec['q_heads'], spec['kv_heads'], (0, spec['batch']), spec['seed'],
                         torch.device('cuda', 0))
    lens = [int(x) for x in data['host_lens'].tolist()]
    pre_k, pre_v = data['k_pool'].clone(), data['v_pool'].clone()
    out = torch.empty_like(data['q'])
    attention.paged_decode_with_append(data['q'], data['k_new'][:, :, 0], data['v_new'][:, :, 0], data['k_pool'],
                                       data['v_pool'], data['block_table'], data['context_lens'],
                                       max_context_len=max(lens), out=out, schedule='stream')
    torch.cuda.synchronize()
    _check_append(spec, data, lens, pre_k, pre_v)
    sequences = range(len(lens)) if len(lens) <= 64 else _extremes_and_stride(lens, 24)
    _check_attention(spec, data, lens, out, sequences)
