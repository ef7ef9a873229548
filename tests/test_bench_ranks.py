"""bench.py's per-rank step times: one collective, every rank's value in rank order (gloo, CPU)."""
import os
import socket

import torch.distributed as dist
import torch.multiprocessing as mp


def _worker(rank, world, port, result_queue):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    import datetime

    import bench
    dist.init_process_group('gloo', rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        result_queue.put((rank, bench.per_rank_values(1.5 * (rank + 1), rank, world, 'cpu')))
    finally:
        dist.destroy_process_group()


def test_every_rank_gets_every_ranks_value_in_rank_order():
    with socket.socket() as sock:
        sock.bind(('127.0.0.1', 0))
        port = sock.getsockname()[1]
    world = 3
    ctx = mp.get_context('spawn')
    queue = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for proc in procs:
        proc.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for proc in procs:
        proc.join(timeout=60)
        assert proc.exitcode == 0
    assert results == {r: [1.5, 3.0, 4.5] for r in range(world)}


def test_one_rank_needs_no_process_group():
    import bench
    assert bench.per_rank_values(2.25, 0, 1, 'cpu') == [2.25]
