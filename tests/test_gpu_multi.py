"""KV-head sharded decode on 2+ GPUs, with the NCCL full-head all-gather.

Each rank runs the decode for its shard of the KV heads (whole GQA groups, or
a batch slice when ranks outnumber KV heads) on its own GPU, then the
full-head output is all-gathered over NCCL and compared with the single-GPU
result and the oracle. Skipped with fewer than two GPUs.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as sock:
        sock.bind(('127.0.0.1', 0))
        return sock.getsockname()[1]


def _worker(rank, world, port, name, result_queue):
    import datetime
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parents[1]
    for path in (root, root / 'micro-vllm_b200'):
        sys.path.insert(0, str(path))
    import numpy as np
    import torch.distributed as dist

    from micro_vllm_b200 import cuda_attention, cuda_paged_cache
    from micro_vllm_b200.sharding import gather_full_heads, kv_head_shard
    from oracle import decode_float
    from tests.golden.cases import make_inputs
    from tests.helpers import assert_attention_close, to_torch

    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    torch.cuda.set_device(rank)
    device = torch.device('cuda', rank)
    dist.init_process_group('nccl', rank=rank, world_size=world, device_id=device,
                            timeout=datetime.timedelta(seconds=120))
    try:
        inputs = make_inputs(name)
        spec = inputs['spec']
        dtype = spec['dtype']
        s = kv_head_shard(rank, world, q_heads=spec['q_heads'], kv_heads=spec['kv_heads'],
                          batch=spec['batch'])
        b0, b1 = s.batch
        k0, k1 = s.kv_heads
        q0, q1 = s.q_heads
        # This rank's page pool holds only its KV heads: [P, Hkv/N, bs, D].
        key_pool = to_torch(np.ascontiguousarray(inputs['key_pool'][:, k0:k1]), dtype, device)
        value_pool = to_torch(np.ascontiguousarray(inputs['value_pool'][:, k0:k1]), dtype, device)
        table = to_torch(inputs['block_table'][b0:b1], None, device)
        lens = to_torch(inputs['context_lens'][b0:b1], None, device)
        key_new = to_torch(np.ascontiguousarray(inputs['key_new'][b0:b1, k0:k1]), dtype, device)
        value_new = to_torch(np.ascontiguousarray(inputs['value_new'][b0:b1, k0:k1]), dtype, device)
        q = to_torch(np.ascontiguousarray(inputs['q'][b0:b1, q0:q1]), dtype, device)
        cuda_paged_cache.write_paged_kv(key_new, value_new, key_pool, value_pool, table,
                                        positions=lens, positions_are_end=True)
        local = cuda_attention.paged_decode_attention(q, key_pool, value_pool, table, lens)
        full = gather_full_heads(local, q_heads=spec['q_heads'], kv_heads=spec['kv_heads'],
                                 batch=spec['batch'])
        torch.cuda.synchronize()
        # Oracle on the full (unsharded) pools after the same append.
        from oracle import append_tokens
        kp, vp = inputs['key_pool'].copy(), inputs['value_pool'].copy()
        append_tokens(kp, vp, inputs['key_new'], inputs['value_new'], inputs['block_table'],
                      inputs['context_lens'].astype(np.int64) - 1)
        expected = decode_float(inputs['q'], kp, vp, inputs['block_table'], inputs['context_lens'],
                                spec['head_dim'] ** -0.5, dtype)
        from tests.helpers import as_float
        assert_attention_close(as_float(full), expected, dtype)
        result_queue.put((rank, 'ok'))
    except Exception as exc:  # reported to the parent, which fails the test
        result_queue.put((rank, repr(exc)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason='two CUDA GPUs required')
@pytest.mark.parametrize('name', ['qwen72b_bf16_small', 'qwen7b_bf16_small'])
def test_kv_head_sharded_decode_matches_the_oracle(name):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, queue)) for r in range(world)]
    for proc in procs:
        proc.start()
    results = dict(queue.get(timeout=300) for _ in procs)
    for proc in procs:
        proc.join(timeout=120)
    assert results == {r: 'ok' for r in range(world)}, results
