"""GPU: the bounded-wait failure path, made to fire without faulting the GPU.

Every wait in this library's kernels gives up after a time limit, raises a
sticky status bit that the host reads (``mv_device_status``) and returns, so
the CUDA context stays usable. ``mv_selftest_wait_timeout`` runs the same
bounded wait on a barrier phase that nothing completes, with a short limit:
the test checks that the wait gives up after at least that limit, that the
status bit is raised and stays raised, that a decode on the same context
afterwards is still correct, and that clearing the status works.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from oracle import decode_float
from tests.golden.cases import make_inputs
from tests.helpers import as_float, assert_attention_close, to_numpy, workload_tensors

pytestmark = pytest.mark.gpu


def _status(lib, device):
    from micro_vllm_b200 import _native
    value = ctypes.c_uint32(0)
    _native.check(lib.mv_device_status(device, ctypes.byref(value)))
    return value.value


def _decode_matches_the_oracle():
    from micro_vllm_b200 import cuda_attention, cuda_paged_cache
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    cuda_paged_cache.write_paged_kv(t['key_new'], t['value_new'], t['key_pool'], t['value_pool'],
                                    t['block_table'], positions=t['context_lens'], positions_are_end=True)
    out = cuda_attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], t['block_table'],
                                                t['context_lens'])
    torch.cuda.synchronize()
    expected = decode_float(inputs['q'], to_numpy(t['key_pool']), to_numpy(t['value_pool']),
                            inputs['block_table'], inputs['context_lens'], 128 ** -0.5, 'bfloat16')
    assert_attention_close(as_float(out), expected, 'bfloat16')
    assert np.isfinite(as_float(out)).all()


def test_a_wait_that_never_completes_gives_up_raises_the_status_and_the_context_stays_usable():
    from micro_vllm_b200 import _native
    lib = _native.library()
    device = torch.cuda.current_device()
    _native.check(lib.mv_clear_device_status(device))
    assert _status(lib, device) == 0
    stream = torch.cuda.current_stream().cuda_stream
    limit_ns = 5_000_000
    torch.cuda.synchronize()
    start = time.perf_counter()
    _native.check(lib.mv_selftest_wait_timeout(limit_ns, stream))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - start
    assert elapsed >= limit_ns * 1e-9
    assert _status(lib, device) == _native.DEVICE_STATUS_WAIT_TIMEOUT

    # The context is intact: the kernels still run and give the right answer;
    # the status bit is sticky until cleared.
    _decode_matches_the_oracle()
    assert _status(lib, device) == _native.DEVICE_STATUS_WAIT_TIMEOUT
    _native.check(lib.mv_clear_device_status(device))
    assert _status(lib, device) == 0
    _decode_matches_the_oracle()
    assert _status(lib, device) == 0


def test_the_self_test_rejects_limits_outside_its_range_without_launching():
    from micro_vllm_b200 import _native
    lib = _native.library()
    device = torch.cuda.current_device()
    _native.check(lib.mv_clear_device_status(device))
    stream = torch.cuda.current_stream().cuda_stream
    for limit in (0, 100_000_001):
        assert lib.mv_selftest_wait_timeout(limit, stream) == 1   # MV_ERR_INVALID_ARGUMENT
        assert b'limit_ns' in lib.mv_last_error()
    torch.cuda.synchronize()
    assert _status(lib, device) == 0


@pytest.mark.parametrize('mode', ['auto', 'simt', 'persistent', 'cluster', 'chunk_tiles', 'append'])
def test_a_page_id_outside_the_pool_raises_its_status_bit(mode):
    """Bounds violations are recorded, not trapped: a used block-table entry
    outside the pool gives NaN rows (or a skipped write) and raises
    MV_DEVICE_STATUS_BAD_PAGE_ID; clean calls raise nothing."""
    from micro_vllm_b200 import _native, cuda_attention, cuda_paged_cache
    lib = _native.library()
    device = torch.cuda.current_device()
    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    kw = {'simt': dict(force_simt=True), 'persistent': dict(persistent=True),
          'cluster': dict(cluster=True)}.get(mode, {})

    def run(table):
        if mode == 'append':
            cuda_paged_cache.write_paged_kv(t['key_new'], t['value_new'], t['key_pool'].clone(),
                                            t['value_pool'].clone(), table, positions=t['context_lens'],
                                            positions_are_end=True)
            return None
        if mode == 'chunk_tiles':
            q = torch.randn(t['q'].shape[0], t['q'].shape[1], 16, t['q'].shape[2], device=t['q'].device,
                            dtype=t['q'].dtype)
            return cuda_attention.paged_chunk_attention(q, t['key_pool'], t['value_pool'], table,
                                                        t['context_lens'].clamp(min=16))
        return cuda_attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], table,
                                                     t['context_lens'], **kw)

    _native.check(lib.mv_clear_device_status(device))
    run(t['block_table'])
    torch.cuda.synchronize()
    assert _status(lib, device) == 0
    lens = inputs['context_lens']
    victim = int(np.argmax(lens))
    table = t['block_table'].clone()
    last = (int(lens[victim]) + 15) // 16 - 1
    table[victim, last] = t['key_pool'].shape[0]           # one past the pool
    out = run(table)
    torch.cuda.synchronize()
    assert _status(lib, device) & _native.DEVICE_STATUS_BAD_PAGE_ID
    if out is not None and mode != 'chunk_tiles':
        values = as_float(out)
        assert np.isnan(values[victim]).all()
        others = [b for b in range(values.shape[0]) if b != victim and lens[b] > 0]
        assert np.isfinite(values[others]).all()
    _native.check(lib.mv_clear_device_status(device))
    assert _status(lib, device) == 0
