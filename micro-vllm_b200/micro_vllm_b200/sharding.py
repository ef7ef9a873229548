"""KV-head sharding of the decode attention layer across GPUs.

Each rank owns whole GQA groups -- a contiguous range of KV heads and the
query heads that read them -- so attention itself needs no communication.
When there are more ranks than KV heads, ranks that share a KV-head range
split the batch instead (a 2-D split: KV heads x sequences), still with no
exchange inside attention. ``gather_full_heads`` all-gathers the per-rank
outputs (NCCL over NVLink, or gloo on CPU) only for callers that need every
head on every rank.
"""
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Shard:
    """The slice of one layer's decode work a rank owns."""

    rank: int
    world: int
    kv_heads: tuple   # [lo, hi) of KV heads
    q_heads: tuple    # [lo, hi) of query heads
    batch: tuple      # [lo, hi) of sequences

    @property
    def num_kv_heads(self):
        return self.kv_heads[1] - self.kv_heads[0]

    @property
    def num_q_heads(self):
        return self.q_heads[1] - self.q_heads[0]

    @property
    def num_seqs(self):
        return self.batch[1] - self.batch[0]


def _split(total, parts, index):
    base, extra = divmod(total, parts)
    lo = index * base + min(index, extra)
    return lo, lo + base + (1 if index < extra else 0)


def kv_head_shard(rank, world, *, q_heads, kv_heads, batch):
    """Shard a [batch, q_heads] decode layer with kv_heads KV heads over `world` ranks."""
    if not 0 <= rank < world:
        raise ValueError('rank must lie in [0, world)')
    if q_heads % kv_heads:
        raise ValueError('query head count must be divisible by KV head count')
    group = q_heads // kv_heads
    if kv_heads % world == 0:
        lo, hi = _split(kv_heads, world, rank)
        return Shard(rank, world, (lo, hi), (lo * group, hi * group), (0, batch))
    if world % kv_heads == 0:
        per_head = world // kv_heads
        head, part = divmod(rank, per_head)
        if batch < per_head:
            raise ValueError('batch too small for the ranks sharing a KV head')
        return Shard(rank, world, (head, head + 1), (head * group, (head + 1) * group),
                     _split(batch, per_head, part))
    raise ValueError('world size must divide, or be a multiple of, the KV head count')


def gather_full_heads(local_out, *, q_heads, kv_heads, batch, group=None, timeout=None):
    """All-gather per-rank outputs [num_seqs, num_q_heads, D] into [batch, q_heads, D].

    Every rank calls this with its own shard's output (one collective, the
    same on every rank). NCCL uses ``all_gather_into_tensor``; other backends
    ``all_gather``. Ragged shards are padded to a common size for the exchange.
    timeout (a ``datetime.timedelta``): the longest this call waits for the
    exchange; past it (a peer that died or never joins) it raises
    RuntimeError instead of waiting on the backend, which does not always
    honour its own timeout when a peer's process is gone. Some backends
    (NCCL) raise from the wait, others (gloo) return False; both give the same
    RuntimeError here. After it the gather may still be queued on the
    communicator and may still write its receive buffer: the caller must
    abort or destroy the process group and discard this call's output before
    any further collective.
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    shards = [kv_head_shard(r, world, q_heads=q_heads, kv_heads=kv_heads, batch=batch)
              for r in range(world)]
    rows = max(s.num_seqs for s in shards)
    cols = max(s.num_q_heads for s in shards)
    dim = local_out.shape[-1]
    padded = local_out.new_zeros((rows, cols, dim))
    padded[:local_out.shape[0], :local_out.shape[1]] = local_out
    if dist.get_backend(group) == 'nccl':
        stacked = local_out.new_empty((world, rows, cols, dim))
        work = dist.all_gather_into_tensor(stacked, padded, group=group, async_op=True)
        pieces = list(stacked.unbind(0))
    else:
        pieces = [torch.empty_like(padded) for _ in range(world)]
        work = dist.all_gather(pieces, padded, group=group, async_op=True)
    if timeout is None:
        work.wait()
    else:
        try:
            done = work.wait(timeout)
        except Exception as exc:  # the backend's own timeout or abort error
            raise RuntimeError(f'full-head gather did not complete within {timeout}: {exc}') from exc
        if not done:
            raise RuntimeError(f'full-head gather did not complete within {timeout}')
    full = local_out.new_empty((batch, q_heads, dim))
    for shard, piece in zip(shards, pieces):
        full[shard.batch[0]:shard.batch[1], shard.q_heads[0]:shard.q_heads[1]] = \
            piece[:shard.num_seqs, :shard.num_q_heads]
    return full
