"""This library's kernels against the reference's own CUDA extensions on B200.

The reference JIT-builds two torch extensions for the hot path
(src/micro_vllm/cuda_attention.py:9-23, cuda_paged_cache.py:9-20);
``oracle/build_ref.py`` compiles them from the reference's sources into
oracle/_ref. Here both implementations run on the same inputs: the
reference's paged decode (``_decode_attention_paged``, one sequence per call,
fp16/fp32 only -- csrc/decode_attention.cpp:147-152) against this library's
batched decode, and the reference's paged write (``write_paged_kv``,
csrc/paged_kv_cache.cpp:96-107) against this library's batched append, which
must be bit-identical. Skipped when oracle/_ref was not built.
"""
import numpy as np
import pytest
import torch

from oracle.build_ref import load
from tests.golden.cases import WORKLOADS, make_inputs
from tests.helpers import workload_tensors

pytestmark = pytest.mark.gpu

REF_ATTN = load('_micro_vllm_decode_attention')
REF_CACHE = load('_micro_vllm_paged_cache')
needs_ref = pytest.mark.skipif(REF_ATTN is None or REF_CACHE is None,
                               reason='reference extensions not built (python oracle/build_ref.py)')

# fp32 and fp16 workloads (the reference kernels take no bf16): the 0.5B
# geometry, the 7B geometry in fp16, and odd shapes from the reference's tests.
CASES = {
    'qwen05b_fp32': 'qwen05b_fp32',
    'qwen05b_fp16': 'qwen05b_fp16',
    'qwen7b_fp16_small': dict(WORKLOADS['qwen7b_bf16_small'], dtype='float16', seed=2102),
    'qwen72b_fp16_small': dict(WORKLOADS['qwen72b_bf16_small'], dtype='float16', seed=5102),
    'edge_bs4_d257_fp16': 'edge_bs4_d257_fp16',
    'edge_bs3_d33_fp32': 'edge_bs3_d33_fp32',
}
# Two implementations, each within the oracle bar of the exact result.
TOLERANCE = {torch.float32: dict(rtol=2e-5, atol=2e-6), torch.float16: dict(rtol=4e-3, atol=4e-3)}


def _table_row(table, b, length, bs):
    return table[b, :-(-length // bs)].to(torch.int64).contiguous()


@needs_ref
@pytest.mark.parametrize('name', list(CASES))
def test_decode_matches_the_reference_kernel(name):
    from micro_vllm_b200 import cuda_attention
    inputs = make_inputs(CASES[name])
    t = workload_tensors(inputs)
    bs = inputs['spec']['block_size']
    ours = cuda_attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], t['block_table'],
                                                 t['context_lens'])
    lens = inputs['context_lens'].tolist()
    for b, length in enumerate(lens):
        theirs = REF_ATTN._decode_attention_paged(t['q'][b:b + 1].unsqueeze(2), t['key_pool'], t['value_pool'],
                                                  _table_row(t['block_table'], b, length, bs), int(length))
        torch.testing.assert_close(ours[b].float(), theirs[0, :, 0].float(), **TOLERANCE[t['q'].dtype])


@needs_ref
@pytest.mark.parametrize('name', ['qwen05b_fp32', 'qwen7b_fp16_small', 'edge_bs3_d33_fp32'])
def test_append_matches_the_reference_kernel_bit_for_bit(name):
    from micro_vllm_b200 import cuda_paged_cache
    inputs = make_inputs(CASES[name])
    t = workload_tensors(inputs)
    bs = inputs['spec']['block_size']
    ref_k, ref_v = t['key_pool'].clone(), t['value_pool'].clone()
    for b, length in enumerate(inputs['context_lens'].tolist()):
        REF_CACHE.write_paged_kv(t['key_new'][b:b + 1], t['value_new'][b:b + 1], ref_k, ref_v,
                                 _table_row(t['block_table'], b, length, bs), int(length) - 1)
    cuda_paged_cache.write_paged_kv(t['key_new'], t['value_new'], t['key_pool'], t['value_pool'],
                                    t['block_table'], positions=t['context_lens'], positions_are_end=True)
    torch.cuda.synchronize()
    assert torch.equal(t['key_pool'].view(torch.uint8), ref_k.view(torch.uint8))
    assert torch.equal(t['value_pool'].view(torch.uint8), ref_v.view(torch.uint8))


@needs_ref
def test_corrupted_page_gives_nan_heads_in_both():
    """An out-of-range page ID: the reference's kernel NaNs the sequence's heads
    (csrc/decode_attention_paged.cu:30-37); so does this library's, and only there."""
    from micro_vllm_b200 import cuda_attention
    inputs = make_inputs(CASES['qwen7b_fp16_small'])    # lengths 1, 17, 300
    inputs['block_table'] = inputs['block_table'].copy()
    inputs['block_table'][2, 5] = inputs['key_pool'].shape[0] + 3
    t = workload_tensors(inputs)
    ours = cuda_attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], t['block_table'],
                                                 t['context_lens'])
    theirs = REF_ATTN._decode_attention_paged(t['q'][2:3].unsqueeze(2), t['key_pool'], t['value_pool'],
                                              _table_row(t['block_table'], 2, 300, 16), 300)
    assert torch.isnan(theirs).all() and torch.isnan(ours[2]).all()
    assert not np.isnan(ours[:2].float().cpu().numpy()).any()
