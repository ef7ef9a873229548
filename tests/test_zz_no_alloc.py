"""The allocation-free decode entry point, called through the C ABI.

Some callers of this decode kernel cannot call cudaMalloc: a plugin whose host
owns every device allocation and hands it only inputs and outputs, or code that
runs while a stream is being captured into a CUDA graph, where allocation is
not allowed. ``mv_paged_decode_noalloc`` serves them with a split-KV scratch
array built into the library. These tests call it directly through ctypes and
check it against the workspace-taking entry point (``mv_paged_decode``, via
``paged_decode_attention``) on the same inputs, twice in a row, at the parity
tolerance the other tests use. This file is collected last on purpose.
"""
import ctypes

import pytest
import torch

from tests.golden.cases import make_inputs
from tests.helpers import as_float, assert_attention_close, workload_tensors

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
                 batch=None, q_heads=None):
    batch = q.shape[0] if batch is None else batch
    q_heads = q.shape[1] if q_heads is None else q_heads
    num_blocks, kv_heads, block_size, dim = k_cache.shape
    if max_context_len is None:
        max_context_len = table.shape[1] * block_size
    return lib.mv_paged_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), v_cache.data_ptr(), num_blocks,
        kv_heads, block_size, dim, table.data_ptr(), INDEX[table.dtype], table.stride(0), table.shape[1],
        lens.data_ptr(), INDEX[lens.dtype], max_context_len, batch, q_heads, dim ** -0.5,
        out.data_ptr(), out.stride(0), out.stride(1), 0, flags, DTYPES[q.dtype],
        torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize('name', ['qwen7b_bf16_small', 'qwen3_8b_bf16_small', 'qwen05b_fp32',
                                  'edge_bs4_d257_fp16'])
def test_noalloc_matches_the_workspace_entry_point_on_two_calls_in_a_row(name):
    from micro_vllm_b200 import cuda_attention, cuda_paged_cache
    lib = library()
    inputs = make_inputs(name)
    dtype = inputs['spec']['dtype']
    t = workload_tensors(inputs)
    cuda_paged_cache.write_paged_kv(t['key_new'], t['value_new'], t['key_pool'], t['value_pool'],
                                    t['block_table'], positions=t['context_lens'], positions_are_end=True)
    reference = cuda_attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'],
                                                      t['block_table'], t['context_lens'])
    torch.cuda.synchronize()
    for _ in range(2):
        out = torch.full_like(reference, float('nan'))
        status = call_noalloc(lib, t['q'], t['key_pool'], t['value_pool'], t['block_table'],
                              t['context_lens'], out)
        assert status == 0, lib.mv_last_error()
        torch.cuda.synchronize()
        assert torch.isfinite(out).all()
        assert_attention_close(as_float(out), as_float(reference), dtype)


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
