"""GPU parity of multi-token chunk attention over pages (``mv_paged_chunk_attention``).

A chunk of T new tokens per sequence, its K/V already appended: token t
attends the first len - (T - 1 - t) tokens. The reference gathers the pages
and runs causal attention (model.py:178-182); the oracle here is the same
math per (sequence, token) over the pages.
"""
import numpy as np
import pytest
import torch

from oracle import decode_float
from tests.golden.cases import make_inputs
from tests.helpers import as_float, assert_attention_close, to_torch, workload_tensors

pytestmark = pytest.mark.gpu

MODES = {'auto': {}, 'simt': dict(force_simt=True), 'rows': dict(kernel='rows'),
         'mma_sync': dict(kernel='mma_sync'), 'split4': dict(pages_per_split=4),
         'rows_split4': dict(pages_per_split=4, kernel='rows'),
         'mma_sync_split4': dict(pages_per_split=4, kernel='mma_sync')}


def _chunk_oracle(inputs, q_np, tokens, dtype):
    """Flatten (sequence, token) into rows: same table row, length len - (T - 1 - t)."""
    lens = inputs['context_lens'].astype(np.int64)
    batch = lens.shape[0]
    rows_q = q_np.transpose(0, 2, 1, 3).reshape(batch * tokens, q_np.shape[1], q_np.shape[3])
    rows_table = np.repeat(inputs['block_table'], tokens, axis=0)
    rows_lens = (lens[:, None] - (tokens - 1 - np.arange(tokens))[None, :]).reshape(-1)
    out = decode_float(rows_q, inputs['key_pool'], inputs['value_pool'], rows_table, rows_lens,
                       q_np.shape[-1] ** -0.5, dtype)
    return out.reshape(batch, tokens, q_np.shape[1], q_np.shape[3]).transpose(0, 2, 1, 3)


@pytest.mark.parametrize('name', ['qwen7b_bf16_small', 'qwen72b_bf16_small', 'qwen05b_fp32',
                                  'edge_bs4_d257_fp16', 'edge_bs64_d64_bf16'])
@pytest.mark.parametrize('tokens', [1, 3, 16])
@pytest.mark.parametrize('mode', list(MODES))
def test_chunk_rows_match_the_oracle(name, tokens, mode):
    from micro_vllm_b200 import cuda_attention
    inputs = make_inputs(name)
    dtype = inputs['spec']['dtype']
    t = workload_tensors(inputs)
    rng = np.random.default_rng(tokens)
    batch, hq, dim = inputs['q'].shape
    from oracle.dtypes import from_float32
    q_np = from_float32(rng.standard_normal((batch, hq, tokens, dim), dtype=np.float32), dtype)
    q = to_torch(q_np, dtype)
    out = cuda_attention.paged_chunk_attention(q, t['key_pool'], t['value_pool'], t['block_table'],
                                               t['context_lens'], **MODES[mode])
    assert out.shape == q.shape
    expected = _chunk_oracle(inputs, q_np, tokens, dtype)
    assert_attention_close(as_float(out), expected, dtype)


def _random_chunk(inputs, tokens, seed):
    from oracle.dtypes import from_float32
    dtype = inputs['spec']['dtype']
    batch, hq, dim = inputs['q'].shape
    rng = np.random.default_rng(seed)
    scale = inputs['spec']['value_scale']
    q_np = from_float32(rng.standard_normal((batch, hq, tokens, dim), dtype=np.float32) * np.float32(scale), dtype)
    return q_np, to_torch(q_np, dtype)


# (workload, tokens, pages_per_split): long chunks whose rows span several
# 64-row query tiles, head_dim 64 and 128, one and several splits per row.
TILE_CASES = [('qwen3_8b_bf16_small', 64, 0), ('qwen3_8b_bf16_small', 100, 8), ('qwen05b_bf16', 48, 0),
              ('qwen05b_fp16', 70, 3), ('qwen72b_bf16_small', 9, 1), ('qwen7b_bf16_small', 130, 0)]


@pytest.mark.parametrize('name, tokens, pps', TILE_CASES)
def test_query_tiles_match_the_oracle_and_the_row_kernel(name, tokens, pps):
    """The tile kernel and the row-per-token kernel both meet the oracle's bar."""
    from micro_vllm_b200 import cuda_attention
    inputs = make_inputs(name)
    dtype = inputs['spec']['dtype']
    t = workload_tensors(inputs)
    q_np, q = _random_chunk(inputs, tokens, 7 + tokens)
    args = (q, t['key_pool'], t['value_pool'], t['block_table'], t['context_lens'])
    tiles = cuda_attention.paged_chunk_attention(*args, pages_per_split=pps)
    rows = cuda_attention.paged_chunk_attention(*args, pages_per_split=pps, kernel='rows')
    mma_sync = cuda_attention.paged_chunk_attention(*args, pages_per_split=pps, kernel='mma_sync')
    expected = _chunk_oracle(inputs, q_np, tokens, dtype)
    assert_attention_close(as_float(tiles), expected, dtype)
    assert_attention_close(as_float(rows), expected, dtype)
    assert_attention_close(as_float(mma_sync), expected, dtype)


@pytest.mark.parametrize('pps', [0, 8])
def test_corrupted_page_poisons_only_the_rows_that_reach_it(pps):
    """A bad page ID poisons exactly the chunk rows whose context covers it
    (rows before it in the same tile stay finite); other sequences are untouched."""
    from micro_vllm_b200 import cuda_attention
    inputs = make_inputs('qwen3_8b_bf16_small')   # lengths 700 and 1029
    inputs['block_table'] = inputs['block_table'].copy()
    num_pages = inputs['key_pool'].shape[0]
    inputs['block_table'][1, 62] = num_pages + 5     # tokens 992..1007 of sequence 1
    inputs['block_table'][0, 43] = -3                # tokens 688..703 of sequence 0
    t = workload_tensors(inputs)
    q_np, q = _random_chunk(inputs, 64, 11)
    out = cuda_attention.paged_chunk_attention(q, t['key_pool'], t['value_pool'], t['block_table'],
                                               t['context_lens'], pages_per_split=pps)
    expected = _chunk_oracle(inputs, q_np, 64, 'bfloat16')
    nan_tokens = np.isnan(expected[1, 0, :, 0])
    assert nan_tokens.any() and not nan_tokens.all()
    assert_attention_close(as_float(out), expected, 'bfloat16')


LONG_SPEC = dict(batch=2, q_heads=8, kv_heads=2, head_dim=64, block_size=16, pool=('factor', 1.25),
                 lens=('fixed', [2100, 1500]), dtype='bfloat16', value_scale=1.0, seed=9101)


@pytest.mark.parametrize('pps', [1, 0])
def test_query_tiles_with_many_splits(pps):
    """132 one-page splits per row (the merge pass combines up to 132 partials),
    and the automatic plan's few long splits."""
    from micro_vllm_b200 import cuda_attention
    inputs = make_inputs(LONG_SPEC)
    t = workload_tensors(inputs)
    q_np, q = _random_chunk(inputs, 8, 5)
    out = cuda_attention.paged_chunk_attention(q, t['key_pool'], t['value_pool'], t['block_table'],
                                               t['context_lens'], pages_per_split=pps)
    assert_attention_close(as_float(out), _chunk_oracle(inputs, q_np, 8, 'bfloat16'), 'bfloat16')


def test_unaligned_query_runs_the_row_kernel_on_the_tile_plan():
    """A query whose element pairs are not 4-byte aligned cannot feed the tile
    kernel; the row-per-token kernel runs on the same splits and workspace."""
    from micro_vllm_b200 import cuda_attention
    from tests.helpers import to_numpy
    inputs = make_inputs('qwen3_8b_bf16_small')
    t = workload_tensors(inputs)
    batch, hq, dim = t['q'].shape
    store = torch.randn(batch, hq, 24, dim + 1, device='cuda').to(torch.bfloat16)
    q = store[..., 1:]                                    # 2-byte offset, odd strides
    out = cuda_attention.paged_chunk_attention(q, t['key_pool'], t['value_pool'], t['block_table'],
                                               t['context_lens'])
    expected = _chunk_oracle(inputs, to_numpy(q.contiguous()), 24, 'bfloat16')
    assert_attention_close(as_float(out), expected, 'bfloat16')


def test_one_token_chunk_equals_decode_bit_for_bit():
    from micro_vllm_b200 import cuda_attention
    t = workload_tensors(make_inputs('qwen7b_bf16_small'))
    q4 = t['q'].unsqueeze(2)
    a = cuda_attention.paged_chunk_attention(q4, t['key_pool'], t['value_pool'], t['block_table'], t['context_lens'])
    b = cuda_attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], t['block_table'],
                                              t['context_lens'])
    assert torch.equal(a[:, :, 0].view(torch.int16), b.view(torch.int16))


def test_strided_chunk_queries_and_outputs():
    from micro_vllm_b200 import cuda_attention
    inputs = make_inputs('qwen72b_bf16_small')
    t = workload_tensors(inputs)
    batch, hq, dim = t['q'].shape
    store = torch.randn(batch, 5, hq + 3, dim, device='cuda').to(torch.bfloat16)
    q = store[:, :, 1:hq + 1].transpose(1, 2)             # [B, Hq, T=5, D], token stride != D
    out_store = torch.full((batch, hq, 5, dim + 8), float('nan'), device='cuda', dtype=torch.bfloat16)
    out = cuda_attention.paged_chunk_attention(q, t['key_pool'], t['value_pool'], t['block_table'],
                                               t['context_lens'], out=out_store[..., :dim])
    assert torch.isnan(out_store[..., dim:]).all()
    from tests.helpers import to_numpy
    expected = _chunk_oracle(inputs, to_numpy(q.contiguous()), 5, 'bfloat16')
    assert_attention_close(as_float(out.contiguous()), expected, 'bfloat16')


def test_two_chunk_prefill_matches_one_prefill():
    from micro_vllm_b200.runtime import prepare_model
    from tests.golden.model_cases import make_prompts, make_weights, model_config
    name = 'tiny_qwen2_fp32'
    weights = {k: torch.from_numpy(v).cuda() for k, v in make_weights(name).items()}
    model = prepare_model(weights, model_config(name))
    prompts = torch.from_numpy(make_prompts(name)).cuda()
    one = model.allocate_cache(prompts.shape[0], 64)
    full = model.prefill(prompts, one)
    two = model.allocate_cache(prompts.shape[0], 64)
    model.prefill(prompts[:, :20], two)
    split = model.prefill(prompts[:, 20:], two)
    torch.testing.assert_close(split, full, rtol=1e-4, atol=1e-4)
    for layer in range(model.num_layers):
        for b in range(prompts.shape[0]):
            ka, va = one.gather(layer, b)
            kb, vb = two.gather(layer, b)
            torch.testing.assert_close(kb, ka, rtol=1e-5, atol=1e-5)
            torch.testing.assert_close(vb, va, rtol=1e-5, atol=1e-5)
