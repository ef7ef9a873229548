"""The allocation-free decode entry point, called through the C ABI.

Some callers of this decode kernel cannot call cudaMalloc: a plugin whose host
owns every device allocation hands it only inputs and outputs, so there is no
workspace to pass and no right to allocate one. ``mv_paged_decode_noalloc``
serves them with a split-KV scratch array built into the library. These tests
call it directly through ctypes, on cases whose plan splits every long
sequence (so the built-in array really carries partial results), twice in a
row (the array keeps the last call's contents), and check each output against
the workspace-taking entry point (``mv_paged_decode``, via
``paged_decode_attention``) and against the oracle, at the parity tolerance
the other tests use.

The file is named to be collected last (pytest collects test files in name
order): a failure here then stops a ``-x`` run only after every other test
has run. Nothing in it depends on running after the others; it also passes
alone in a fresh process.
"""
import ctypes

import pytest
import torch

from oracle import decode_float
from tests.golden.cases import make_inputs
from tests.helpers import as_float, assert_attention_close, to_numpy, workload_tensors

pytestmark = pytest.mark.gpu

_i32, _i64, _u32, _vp, _f32 = ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_float
NOALLOC_ARGTYPES = [_vp, _i64, _i64, _vp, _vp, _i64, _i32, _i32, _i32, _vp, _i32, _i64, _i64, _vp, _i32,
                    _i64, _i32, _i32, _f32, _vp, _i64, _i64, _i32, _u32, _i32, _vp]
DTYPES = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}
INDEX = {torch.int32: 0, torch.int64: 1}


def library():
    from micro_vllm_b200 import _native
    lib = _native.library()
    fn = lib.mv_paged_decode_noalloc
    fn.argtypes = NOALLOC_ARGTYPES
    fn.restype = ctypes.c_int
    return lib


def call_noalloc(lib, q, k_cache, v_cache, table, lens, out, *, max_context_len=None, flags=0,
                 pages_per_split=0, batch=None, q_heads=None):
    batch = q.shape[0] if batch is None else batch
    q_heads = q.shape[1] if q_heads is None else q_heads
    num_blocks, kv_heads, block_size, dim = k_cache.shape
    if max_context_len is None:
        max_context_len = table.shape[1] * block_size
    return lib.mv_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), num_blocks,
        kv_heads, block_size, dim, table.data_ptr(), INDEX[table.dtype], table.stride(0), table.shape[1],
        lens.data_ptr(), INDEX[lens.dtype], max_context_len, batch, q_heads, dim ** -0.5,
        out.data_ptr(), out.stride(0), out.stride(1), pages_per_split, flags, DTYPES[q.dtype],
        torch.cuda.current_stream().cuda_stream)


def _misaligned_copy(pool):
    """The same pages, one element past a 16-byte boundary (no TMA: the CUDA-core plan)."""
    flat = torch.empty(pool.numel() + 1, dtype=pool.dtype, device=pool.device)
    view = flat[1:].view(pool.shape)
    view.copy_(pool)
    return view


# (workload, pages_per_split, misaligned caches): every plan has more than one split.
CASES = {
    'qwen7b_bf16_small': ('qwen7b_bf16_small', 0, False),          # tensor-core split grid
    'qwen7b_bf16_small_pps1': ('qwen7b_bf16_small', 1, False),     # one page per split
    'qwen3_8b_bf16_small': ('qwen3_8b_bf16_small', 0, False),
    'qwen7b_bf16_small_misaligned': ('qwen7b_bf16_small', 0, True),  # CUDA-core plan, its own split sizes
    'qwen05b_fp32': ('qwen05b_fp32', 0, False),                    # CUDA-core kernel
    'edge_bs4_d257_fp16': ('edge_bs4_d257_fp16', 0, False),
}


@pytest.mark.parametrize('case', list(CASES))
def test_noalloc_matches_the_workspace_entry_point_and_the_oracle_on_two_calls_in_a_row(case):
    from micro_vllm_b200 import cuda_attention, cuda_paged_cache
    name, pps, misaligned = CASES[case]
    lib = library()
    inputs = make_inputs(name)
    dtype = inputs['spec']['dtype']
    t = workload_tensors(inputs)
    cuda_paged_cache.write_paged_kv(t['key_new'], t['value_new'], t['key_pool'], t['value_pool'],
                                    t['block_table'], positions=t['context_lens'], positions_are_end=True)
    key_pool, value_pool = t['key_pool'], t['value_pool']
    if misaligned:
        key_pool, value_pool = _misaligned_copy(key_pool), _misaligned_copy(value_pool)
    batch, q_heads = t['q'].shape[:2]
    bound = t['block_table'].shape[1] * key_pool.shape[2]
    path, _, splits = cuda_attention.paged_decode_plan(q_heads, key_pool, bound, batch=batch,
                                                       pages_per_split=pps)
    assert splits > 1, 'the case must split sequences so the built-in scratch is used'
    assert (path == 'simt') == (misaligned or dtype == 'float32' or inputs['spec']['head_dim'] == 257)
    reference = cuda_attention.paged_decode_attention(t['q'], key_pool, value_pool, t['block_table'],
                                                      t['context_lens'], pages_per_split=pps)
    torch.cuda.synchronize()
    expected = decode_float(inputs['q'], to_numpy(t['key_pool']), to_numpy(t['value_pool']),
                            inputs['block_table'], inputs['context_lens'], inputs['spec']['head_dim'] ** -0.5,
                            dtype)
    for _ in range(2):
        out = torch.full_like(reference, float('nan'))
        status = call_noalloc(lib, t['q'], key_pool, value_pool, t['block_table'], t['context_lens'], out,
                              pages_per_split=pps)
        assert status == 0, lib.mv_last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert_attention_close(as_float(out), as_float(reference), dtype)
        assert_attention_close(as_float(out), expected, dtype)


def test_noalloc_rejects_calls_beyond_its_scratch_and_the_fused_merge_flag():
    lib = library()
    q = torch.zeros(256, 64, 128, dtype=torch.bfloat16, device='cuda')
    pool = torch.zeros(4, 8, 16, 128, dtype=torch.bfloat16, device='cuda')
    table = torch.zeros(256, 2048, dtype=torch.int32, device='cuda')
    lens = torch.ones(256, dtype=torch.int32, device='cuda')
    out = torch.empty_like(q)
    status = call_noalloc(lib, q, pool, pool, table, lens, out, max_context_len=32768)
    assert status == 2
    assert b'scratch' in lib.mv_last_error()
    small = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(small)
    status = call_noalloc(lib, t['q'], t['key_pool'], t['value_pool'], t['block_table'],
                          t['context_lens'], torch.empty_like(t['q']), flags=4)
    assert status == 2
    assert b'FUSED_MERGE' in lib.mv_last_error()


def test_noalloc_sizes_its_scratch_with_the_plan_of_misaligned_caches():
    """16 sequences of up to 16,384 tokens, 64/4 heads of 256: aligned caches plan a
    first split of 128 pages then 64-page splits (15 splits, 16.05 MB of scratch:
    fits the 16 MiB array); misaligned ones take the CUDA-core plan of uniform
    64-page splits (16 splits, 17.1 MB: does not fit). The misaligned call is
    rejected with the scratch message, before any launch; the aligned one runs."""
    from micro_vllm_b200 import cuda_attention
    lib = library()
    q = torch.zeros(16, 64, 256, dtype=torch.bfloat16, device='cuda')
    pool = torch.zeros(8, 4, 16, 256, dtype=torch.bfloat16, device='cuda')
    table = torch.zeros(16, 1024, dtype=torch.int32, device='cuda')
    lens = torch.ones(16, dtype=torch.int32, device='cuda')
    assert cuda_attention.paged_decode_plan(64, pool, 16384, batch=16) == ('tma_mma', 64, 15)
    misaligned = _misaligned_copy(pool)
    assert cuda_attention.paged_decode_plan(64, misaligned, 16384, batch=16) == ('simt', 64, 16)
    status = call_noalloc(lib, q, misaligned, misaligned, table, lens, torch.empty_like(q),
                          max_context_len=16384)
    assert status == 2
    assert b'scratch' in lib.mv_last_error()
    out = torch.full_like(q, float('nan'))
    status = call_noalloc(lib, q, pool, pool, table, lens, out, max_context_len=16384)
    assert status == 0, lib.mv_last_error()
    torch.cuda.synchronize()
    assert torch.equal(out, torch.zeros_like(out))     # zero values everywhere: zero output
