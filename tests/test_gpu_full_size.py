"""GPU parity at the benchmark's own sizes, with the benchmark's own launch plan.

``bench.py`` times one decode step -- append this step's K/V row of every
sequence, then paged decode attention over the whole context, in one call
(``paged_decode_with_append``) -- on full-size workloads built on the device
by ``tests/golden/workloads.make_workload``. These tests run that same call on
those same inputs (same seeds, same KV-head shard geometry as ``bench.py
--scaling strong`` gives a rank) and check it against the oracle:

* the launch plan ``paged_decode_plan`` reports for the call is the one the
  bench line reports (asserted exactly for each workload);
* the append: the page each sequence wrote equals, bit for bit, the oracle's
  append of that row into the page's pre-step contents, and every other page
  of both pools is unchanged;
* attention: every checked sequence's output against the oracle's fp32 math
  on the bf16 inputs (``decode_float`` over that sequence's post-step pages),
  within the bf16 bar of 2e-2 max-abs.

The Qwen3-8B long-context workload reaches 131,072 tokens (8,192 pages) per
sequence with 1% of K rows scaled x8; the Qwen2.5-72B workload is batch 256
with lognormal lengths up to 32,768 tokens. The oracle runs per sequence in
fp32 to bound host memory.
"""
import numpy as np
import pytest
import torch

from oracle import append_tokens, decode_float
from tests.golden.cases import array_digest
from tests.golden.workloads import WORKLOADS, make_workload
from tests.helpers import as_float, assert_attention_close, to_numpy

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _shard(spec, world, rank):
    from micro_vllm_b200.sharding import kv_head_shard
    if world == 1:
        return spec['q_heads'], spec['kv_heads'], (0, spec['batch'])
    shard = kv_head_shard(rank, world, q_heads=spec['q_heads'], kv_heads=spec['kv_heads'],
                          batch=spec['batch'])
    return shard.num_q_heads, shard.num_kv_heads, shard.batch


def _bits(tensor):
    return tensor.view(torch.int16) if tensor.element_size() == 2 else tensor.view(torch.int32)


def _run_bench_step(name, world, rank):
    """The bench's one-call step on the bench's inputs; returns everything the checks need."""
    from micro_vllm_b200 import cuda_attention

    spec = WORKLOADS[name]
    q_heads, kv_heads, batch_slice = _shard(spec, world, rank)
    device = torch.device('cuda', 0)
    data = make_workload(spec, q_heads, kv_heads, batch_slice, spec['seed'], device)
    lens = [int(x) for x in data['host_lens'].tolist()]
    max_len = max(lens)
    plan = cuda_attention.paged_decode_plan(q_heads, data['k_pool'], max_len, batch=len(lens))
    pre_k, pre_v = data['k_pool'].clone(), data['v_pool'].clone()
    out = torch.empty_like(data['q'])
    cuda_attention.paged_decode_with_append(
        data['q'], data['k_new'][:, :, 0], data['v_new'][:, :, 0], data['k_pool'], data['v_pool'],
        data['block_table'], data['context_lens'], max_context_len=max_len, out=out)
    torch.cuda.synchronize()
    return spec, data, lens, plan, pre_k, pre_v, out


def _check_append(spec, data, lens, pre_k, pre_v):
    """The written page of each sequence against the oracle's append; all else unchanged."""
    bs = spec['block_size']
    batch = len(lens)
    table = data['host_table'].to(torch.int64)
    last_logical = torch.tensor([(n - 1) // bs for n in lens], dtype=torch.int64)
    last = table[torch.arange(batch), last_logical]
    assert len(set(last.tolist())) == batch        # permutation slices: one written page per sequence
    last_dev = last.to(data['k_pool'].device)
    local_table = np.full((batch, int(last_logical.max()) + 1), -1, dtype=np.int64)
    local_table[np.arange(batch), last_logical.numpy()] = np.arange(batch)
    expected_k = to_numpy(pre_k.index_select(0, last_dev))
    expected_v = to_numpy(pre_v.index_select(0, last_dev))
    append_tokens(expected_k, expected_v, to_numpy(data['k_new']), to_numpy(data['v_new']), local_table,
                  np.asarray(lens, dtype=np.int64) - 1)
    assert array_digest(to_numpy(data['k_pool'].index_select(0, last_dev))) == array_digest(expected_k)
    assert array_digest(to_numpy(data['v_pool'].index_select(0, last_dev))) == array_digest(expected_v)
    untouched = torch.ones(pre_k.shape[0], dtype=torch.bool, device=pre_k.device)
    untouched[last_dev] = False
    assert torch.equal(_bits(data['k_pool'][untouched]), _bits(pre_k[untouched]))
    assert torch.equal(_bits(data['v_pool'][untouched]), _bits(pre_v[untouched]))


def _check_attention(spec, data, lens, out, sequences):
    """Each listed sequence's output against the oracle over its own post-step pages."""
    bs, dim, dtype = spec['block_size'], spec['head_dim'], spec['dtype']
    q_host = to_numpy(data['q'])
    out_host = as_float(out)
    worst = 0.0
    for b in sequences:
        n = -(-lens[b] // bs)
        ids = data['host_table'][b, :n].to(torch.int64).to(data['k_pool'].device)
        k_pages = to_numpy(data['k_pool'].index_select(0, ids))
        v_pages = to_numpy(data['v_pool'].index_select(0, ids))
        expected = decode_float(q_host[b:b + 1], k_pages, v_pages, np.arange(n, dtype=np.int64)[None],
                                np.asarray([lens[b]]), dim ** -0.5, dtype, accum=np.float32)
        assert np.isfinite(expected).all()
        assert_attention_close(out_host[b:b + 1], expected, dtype)
        worst = max(worst, float(np.max(np.abs(out_host[b:b + 1] - expected))))
    return worst


def _extremes_and_stride(lens, count):
    """The shortest and longest sequences plus an even spread, ``count`` in all."""
    order = sorted(range(len(lens)), key=lambda b: lens[b])
    picked = {order[0], order[-1]}
    step = max(1, len(lens) // max(1, count - 2))
    picked.update(range(0, len(lens), step))
    return sorted(picked)[:max(count, 2)] if count < len(lens) else list(range(len(lens)))


def test_qwen7b_headline_step_full_size_with_the_bench_plan():
    """Batch 64, 28/4 heads, 1k-4k tokens: the headline workload, every sequence."""
    spec, data, lens, plan, pre_k, pre_v, out = _run_bench_step('qwen7b_bf16', 1, 0)
    max_pages = -(-max(lens) // 16)
    assert max_pages > 128
    # The bench's plan: a first split of 128 pages, a second of 64, then 16-page splits
    # (6 splits at up to 256 pages).
    assert plan == ('tma_mma', 64, 2 + -(-(max_pages - 192) // 16))
    assert plan[2] == 6
    _check_append(spec, data, lens, pre_k, pre_v)
    worst = _check_attention(spec, data, lens, out, range(len(lens)))
    print(f'qwen7b_bf16 full size: plan {plan}, max abs err {worst:.3e}')


def test_qwen3_8b_long_context_full_size_every_sequence():
    """Batch 8, 32/8 heads, 32k-131k tokens, 1% of K rows x8: many splits per sequence."""
    spec, data, lens, plan, pre_k, pre_v, out = _run_bench_step('qwen3_8b_long_bf16', 1, 0)
    max_pages = -(-max(lens) // 16)
    assert max(lens) > 100_000 and min(lens) >= 32768
    assert plan == ('tma_mma', 128, -(-max_pages // 128))
    _check_append(spec, data, lens, pre_k, pre_v)
    worst = _check_attention(spec, data, lens, out, range(len(lens)))
    print(f'qwen3_8b_long_bf16 full size: plan {plan}, max abs err {worst:.3e}')


def test_qwen72b_batch_256_lognormal_full_size():
    """Batch 256, 64/8 heads, lognormal lengths clipped to [16, 32768]: every sequence."""
    spec, data, lens, plan, pre_k, pre_v, out = _run_bench_step('qwen72b_bf16', 1, 0)
    max_pages = -(-max(lens) // 16)
    assert plan == ('tma_mma', 128, -(-max_pages // 128))
    assert plan[2] > 1
    _check_append(spec, data, lens, pre_k, pre_v)
    worst = _check_attention(spec, data, lens, out, range(len(lens)))
    print(f'qwen72b_bf16 full size: plan {plan}, max abs err {worst:.3e}')


@pytest.mark.parametrize('name,world,rank', [
    ('qwen3_8b_long_bf16', 8, 7),    # one KV head (4 query heads) of the long-context layer
    ('qwen3_8b_long_bf16', 2, 0),    # four KV heads
    ('qwen72b_bf16', 8, 0),          # one KV head (8 query heads), batch 256
    ('qwen72b_bf16', 4, 3),          # two KV heads
    ('qwen7b_bf16', 8, 5),           # KV head 2 of 4, batch half 2 of 2 (ranks outnumber heads)
])
def test_kv_head_shards_of_the_strong_scaling_runs(name, world, rank):
    """The slice a rank of ``bench.py --gpus N --scaling strong`` computes, on one GPU."""
    spec, data, lens, plan, pre_k, pre_v, out = _run_bench_step(name, world, rank)
    assert plan[0] == 'tma_mma' and plan[2] > 1
    _check_append(spec, data, lens, pre_k, pre_v)
    sequences = _extremes_and_stride(lens, 24)
    worst = _check_attention(spec, data, lens, out, sequences)
    print(f'{name} shard {rank}/{world}: {data["q"].shape[1]}/{data["k_pool"].shape[1]} heads, '
          f'batch {len(lens)}, plan {plan}, {len(sequences)} sequences checked, max abs err {worst:.3e}')


def test_qwen7b_fused_merge_matches_the_merge_pass_bit_for_bit():
    """The opt-in fused merge (the last split CTA of each segment merges it, a
    warp per output row) on the headline workload: the same bits as the
    default merge pass. The append is idempotent (the same row to the same
    slot), so the second call runs on the first call's pools."""
    from micro_vllm_b200 import cuda_attention

    spec, data, lens, plan, pre_k, pre_v, out = _run_bench_step('qwen7b_bf16', 1, 0)
    k_after, v_after = data['k_pool'].clone(), data['v_pool'].clone()
    fused = torch.empty_like(out)
    cuda_attention.paged_decode_with_append(
        data['q'], data['k_new'][:, :, 0], data['v_new'][:, :, 0], data['k_pool'], data['v_pool'],
        data['block_table'], data['context_lens'], max_context_len=max(lens), out=fused, fused_merge=True)
    torch.cuda.synchronize()
    assert torch.equal(_bits(fused), _bits(out))
    assert torch.equal(_bits(data['k_pool']), _bits(k_after))
    assert torch.equal(_bits(data['v_pool']), _bits(v_after))


def test_qwen7b_two_call_step_matches_the_one_call_step_bit_for_bit():
    """The two-call form of the headline step: the append kernel, then the decode.

    The decode is launched with programmatic dependent launch while the append
    kernel still runs, and its first CTAs prefetch pages into L2 -- among them
    the last page of every sequence, which the append kernel is writing -- before
    they wait for it. Pools and output must equal the one-call step's bit for bit.
    """
    from micro_vllm_b200 import cuda_attention, cuda_paged_cache

    spec, data, lens, plan, pre_k, pre_v, out = _run_bench_step('qwen7b_bf16', 1, 0)
    k_one, v_one = data['k_pool'].clone(), data['v_pool'].clone()
    data['k_pool'].copy_(pre_k)
    data['v_pool'].copy_(pre_v)
    two = torch.empty_like(out)
    cuda_paged_cache.write_paged_kv(data['k_new'], data['v_new'], data['k_pool'], data['v_pool'],
                                    data['block_table'], positions=data['context_lens'], positions_are_end=True)
    cuda_attention.paged_decode_attention(data['q'], data['k_pool'], data['v_pool'], data['block_table'],
                                          data['context_lens'], max_context_len=max(lens), out=two)
    torch.cuda.synchronize()
    assert torch.equal(_bits(data['k_pool']), _bits(k_one))
    assert torch.equal(_bits(data['v_pool']), _bits(v_one))
    assert torch.equal(_bits(two), _bits(out))
