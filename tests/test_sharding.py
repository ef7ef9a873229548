"""KV-head sharding: layout math, and the full-head all-gather over 2 and 4 gloo ranks on CPU."""
import os

import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st
import torch.distributed as dist
import torch.multiprocessing as mp

from micro_vllm_b200.sharding import gather_full_heads, kv_head_shard


@pytest.mark.parametrize('world', [1, 2, 4, 8])
@pytest.mark.parametrize('q_heads, kv_heads, batch', [(28, 4, 64), (32, 8, 8), (64, 8, 256),
                                                      (14, 2, 4), (12, 2, 32)])
def test_shards_cover_every_head_and_sequence_once(world, q_heads, kv_heads, batch):
    if kv_heads % world and world % kv_heads:
        with pytest.raises(ValueError):
            kv_head_shard(0, world, q_heads=q_heads, kv_heads=kv_heads, batch=batch)
        return
    owner = torch.zeros(batch, q_heads, dtype=torch.int64)
    group = q_heads // kv_heads
    for rank in range(world):
        s = kv_head_shard(rank, world, q_heads=q_heads, kv_heads=kv_heads, batch=batch)
        # whole GQA groups only: the query heads are exactly the group of the KV heads
        assert s.q_heads == (s.kv_heads[0] * group, s.kv_heads[1] * group)
        owner[s.batch[0]:s.batch[1], s.q_heads[0]:s.q_heads[1]] += 1
    assert (owner == 1).all()


@settings(max_examples=300, deadline=None)
@given(world=st.integers(1, 16), kv_heads=st.integers(1, 16), group=st.integers(1, 8),
       batch=st.integers(1, 300))
def test_shards_partition_any_valid_layout_in_balanced_slices(world, kv_heads, group, batch):
    q_heads = kv_heads * group
    if kv_heads % world and world % kv_heads:
        with pytest.raises(ValueError):
            kv_head_shard(0, world, q_heads=q_heads, kv_heads=kv_heads, batch=batch)
        return
    if kv_heads % world and batch < world // kv_heads:
        with pytest.raises(ValueError, match='batch too small'):
            kv_head_shard(0, world, q_heads=q_heads, kv_heads=kv_heads, batch=batch)
        return
    shards = [kv_head_shard(r, world, q_heads=q_heads, kv_heads=kv_heads, batch=batch)
              for r in range(world)]
    owner = torch.zeros(batch, q_heads, dtype=torch.int64)
    for s in shards:
        assert s.q_heads == (s.kv_heads[0] * group, s.kv_heads[1] * group)
        owner[s.batch[0]:s.batch[1], s.q_heads[0]:s.q_heads[1]] += 1
    assert (owner == 1).all()
    # Balanced: per-rank work differs by at most one KV head or one sequence.
    units = [s.num_kv_heads * s.num_seqs for s in shards]
    assert max(s.num_kv_heads for s in shards) - min(s.num_kv_heads for s in shards) <= 1
    assert max(s.num_seqs for s in shards) - min(s.num_seqs for s in shards) <= 1
    assert sum(units) == kv_heads * batch


def test_rejects_bad_ranks_and_head_counts():
    with pytest.raises(ValueError):
        kv_head_shard(2, 2, q_heads=28, kv_heads=4, batch=64)
    with pytest.raises(ValueError):
        kv_head_shard(0, 3, q_heads=28, kv_heads=4, batch=64)
    with pytest.raises(ValueError):
        kv_head_shard(0, 2, q_heads=27, kv_heads=4, batch=64)


def _gather_worker(rank, world, port, q_heads, kv_heads, batch, timeout_s, result_queue):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    import datetime
    dist.init_process_group('gloo', rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        full = torch.arange(batch * q_heads * 3, dtype=torch.float32).reshape(batch, q_heads, 3)
        s = kv_head_shard(rank, world, q_heads=q_heads, kv_heads=kv_heads, batch=batch)
        local = full[s.batch[0]:s.batch[1], s.q_heads[0]:s.q_heads[1]].clone()
        timeout = None if timeout_s is None else datetime.timedelta(seconds=timeout_s)
        gathered = gather_full_heads(local, q_heads=q_heads, kv_heads=kv_heads, batch=batch,
                                     timeout=timeout)
        result_queue.put((rank, bool(torch.equal(gathered, full))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('world, q_heads, kv_heads, batch, timeout_s',
                         [(2, 28, 4, 6, None), (2, 14, 1, 5, None), (2, 28, 4, 6, 60),
                          (4, 12, 2, 7, None)])
def test_gather_full_heads_over_gloo_ranks(world, q_heads, kv_heads, batch, timeout_s):
    import socket
    with socket.socket() as sock:
        sock.bind(('127.0.0.1', 0))
        port = sock.getsockname()[1]
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    procs = [ctx.Process(target=_gather_worker, args=(r, world, port, q_heads, kv_heads, batch, timeout_s, queue))
             for r in range(world)]
    for proc in procs:
        proc.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for proc in procs:
        proc.join(timeout=60)
        assert proc.exitcode == 0
    assert results == {r: True for r in range(world)}


def _report(result_queue, item, code):
    # Queue.put hands the item to a feeder thread; flush it to the pipe before
    # os._exit, which would otherwise end the process with the item unsent.
    result_queue.put(item)
    result_queue.close()
    result_queue.join_thread()
    os._exit(code)


def _failure_worker(rank, world, port, mode, result_queue):
    """Rank 1 fails before the full-head gather (dies, or stalls and never
    joins); rank 0 reports how its gather ended."""
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    import datetime
    import time
    try:
        # A generous timeout for the rendezvous (process start-up is slow on a
        # busy host), a short one for the group the gather runs on.
        dist.init_process_group('gloo', rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120))
        group = dist.new_group(ranks=list(range(world)), timeout=datetime.timedelta(seconds=5))
        dist.barrier()   # both ranks are set up before rank 1 fails
    except Exception as exc:  # noqa: BLE001 - reported, the test fails on it
        _report(result_queue, ('setup failed: ' + type(exc).__name__, 0.0), 1)
    full = torch.arange(4 * 28 * 3, dtype=torch.float32).reshape(4, 28, 3)
    s = kv_head_shard(rank, world, q_heads=28, kv_heads=4, batch=4)
    local = full[s.batch[0]:s.batch[1], s.q_heads[0]:s.q_heads[1]].clone()
    if rank == 1:
        if mode == 'dies':
            os._exit(3)
        time.sleep(120)          # stalls: the test ends this process
        os._exit(0)
    start = time.monotonic()
    try:
        gather_full_heads(local, q_heads=28, kv_heads=4, batch=4, group=group,
                          timeout=datetime.timedelta(seconds=10))
        outcome = 'completed'
    except Exception as exc:  # noqa: BLE001 - any error is the expected outcome
        outcome = type(exc).__name__
    _report(result_queue, (outcome, time.monotonic() - start), 0)


@pytest.mark.parametrize('mode', ['dies', 'stalls'])
def test_a_failed_rank_ends_the_full_head_gather_with_an_error_not_a_hang(mode):
    """Host-side failure detection: a peer that exits or never joins makes the
    surviving rank's gather raise within the process group's timeout."""
    import socket
    with socket.socket() as sock:
        sock.bind(('127.0.0.1', 0))
        port = sock.getsockname()[1]
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    procs = [ctx.Process(target=_failure_worker, args=(r, 2, port, mode, queue)) for r in range(2)]
    for proc in procs:
        proc.start()
    try:
        outcome, elapsed = queue.get(timeout=180)
    finally:
        for proc in procs:
            if proc.is_alive():
                proc.terminate()
            proc.join(timeout=30)
    assert outcome != 'completed' and not outcome.startswith('setup failed'), outcome
    assert elapsed < 60
