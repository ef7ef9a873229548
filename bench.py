#!/usr/bin/env python
"""Benchmark: one decode step of one paged GQA attention layer on B200.

A step is the hot path over one batch: append this step's K/V token for every
sequence into its page and run paged decode attention over the whole context.
By default the step is one call, paged_decode_with_append (the decode kernel
writes each sequence's new row into the page it attends); ``--step separate``
times the two-call form, write_paged_kv then paged_decode_attention, and
every run also reports that form's time beside the headline. Workload: Qwen2.5-7B decode
geometry -- batch 64, 28 query / 4 KV heads, head_dim 128, bf16, context
lengths uniform in [1024, 4096], 16-token pages in a randomly permuted pool
1.25x the pages in use, q/K/V ~ 0.5 N(0,1), scale 128^-1/2. Seeded synthetic
data; the KV pool (~0.42 GB per GPU) is larger than the 126 MB L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Prints ONE JSON line on rank 0. ``value`` is whole-job achieved HBM GB/s by
the path's algorithmic bytes (K and V read once, q and out, page indices,
lengths, and the append's read+write), measured with CUDA events around K
steps run as replays of a CUDA graph of 8 back-to-back steps (a serving loop
replays one graph per decode step of all its layers; ``ms_per_step_single_replay``
gives the one-step-per-replay figure beside it), max over ranks. ``e2e`` is the same metric
through the public Python API with this step's inputs copied from pinned host
memory and the output copied back inside the timed region.

Multi-GPU (weak scaling, no collective on the data path): KV-head sharding,
every rank owns a 4-KV-head (7-query-head-group) slice of an N x wider layer
over the same batch, i.e. one config-sized shard per GPU. ``--scaling strong``
instead splits the fixed single-layer workload by KV head (and by batch once
ranks outnumber KV heads).

``--impl reference`` times the reference's CPU path for the same workload
(gather + causal attention + append, restated by the oracle) on the host cores.
"""
import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _path in (ROOT, ROOT / 'micro-vllm_b200'):
    if str(_path) not in sys.path:
        sys.path.insert(0, str(_path))

from tests.golden.workloads import WORKLOADS, make_workload  # noqa: E402

METRIC = 'paged decode attn achieved HBM GB/s (% of B200 peak); decode tokens/s'
DEFAULT_WORKLOAD = 'qwen7b_bf16'
FALLBACK_HBM_GBS = 6650.0
# dram__bytes_read.sum + dram__bytes_write.sum of one step's kernels on this workload, from
# one ncu capture each: paged_decode_mma_kernel with the append fused (329.85 MB + 5.37 MB,
# profiles/paged_decode_mma_qwen7b_bf16.md) + paged_decode_merge_warp_kernel (2.07 MB read with
# ncu's cold caches, profiles/paged_decode_merge_warp_qwen7b_bf16.md).
NCU_TRAFFIC_BYTES = {('qwen7b_bf16', 'tma_mma'): 330_466_048 + 4_808_192 + 2_067_456}
# Kernels of one one-call step by plan path (the roofline's dominant kernel and the merge pass).
STEP_KERNELS = {
    'tma_mma': 'paged_decode_mma_kernel (append fused) + paged_decode_merge_warp_kernel',
    'tma_mma_stream': 'paged_decode_stream_kernel (append fused) + paged_decode_merge_warp_kernel',
}
TRAFFIC_SOURCES = {
    'tma_mma': ('ncu dram__bytes_read.sum + dram__bytes_write.sum of one step: paged_decode_mma_kernel (append '
                'fused) + paged_decode_merge_warp_kernel (profiles/paged_decode_mma_qwen7b_bf16.md, '
                'profiles/paged_decode_merge_warp_qwen7b_bf16.md)'),
}
L2_BYTES = 126 * 1024 * 1024
KERNEL_CALLS = 8


def parse_args(argv=None):
    parser = argparse.ArgumentParser(description=__doc__.split('\n')[0])
    parser.add_argument('--gpus', type=int, default=1)
    parser.add_argument('--steps', type=int, default=2000)
    parser.add_argument('--warmup', type=int, default=20)
    parser.add_argument('--impl', choices=('ours', 'reference'), default='ours')
    parser.add_argument('--workload', default=DEFAULT_WORKLOAD)
    parser.add_argument('--scaling', choices=('weak', 'strong'), default='weak')
    parser.add_argument('--cpu-seconds', type=float, default=12.0,
                        help='wall-clock budget of the CPU baseline sample')
    parser.add_argument('--no-cpu-baseline', action='store_true')
    parser.add_argument('--no-strong-scaling', action='store_true',
                        help='skip the strong-scaling records (profiling runs: only the headline workload on the device)')
    parser.add_argument('--pages-per-split', type=int, default=0)
    parser.add_argument('--kernels', default='',
                        help='kernels_qwen15b workload: time only the entries whose names contain this text')
    parser.add_argument('--nvtx-steps', type=int, default=0,
                        help='generation workload: run prefill and this many eager decode steps inside NVTX '
                             'ranges "prefill" and "decode" (for a profiler launch list), print nothing else')
    parser.add_argument('--step', choices=('fused', 'separate'), default='fused',
                        help='one-call append + attention (default) or the append kernel then attention')
    return parser.parse_args(argv)


# ----------------------------------------------------------------- setup

def init_distributed(args):
    import torch
    world = int(os.environ.get('WORLD_SIZE', '1'))
    rank = int(os.environ.get('RANK', '0'))
    local_rank = int(os.environ.get('LOCAL_RANK', '0'))
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit('--gpus N > 1 needs torchrun --nproc-per-node N')
    if world > 1:
        import datetime
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device('cuda', local_rank))
    return rank, world, local_rank


def per_rank_values(value, rank, world, device):
    """Every rank's `value` (a float) in rank order, on every rank.

    One all-reduce (a sum over slots that only their own rank fills); every
    rank calls it at the same point, as with any collective.
    """
    import torch
    import torch.distributed as dist

    slots = torch.zeros(world, dtype=torch.float64, device=device)
    slots[rank] = value
    if world > 1:
        dist.all_reduce(slots, op=dist.ReduceOp.SUM)
    return slots.tolist()


def peak_hbm():
    path = ROOT / 'MEASURED_PEAKS.json'
    try:
        data = json.loads(path.read_text())
        return float(data['hbm_gbs']), 'measured'
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, 'fallback'


def local_geometry(spec, rank, world, scaling):
    """(q_heads, kv_heads, batch slice) this rank computes."""
    from micro_vllm_b200.sharding import kv_head_shard
    if world == 1 or scaling == 'weak':
        return spec['q_heads'], spec['kv_heads'], (0, spec['batch'])
    shard = kv_head_shard(rank, world, q_heads=spec['q_heads'], kv_heads=spec['kv_heads'],
                          batch=spec['batch'])
    return shard.num_q_heads, shard.num_kv_heads, shard.batch


def step_bytes(spec, lens, q_heads, kv_heads):
    """Algorithmic bytes of one step (decode + append) for this rank's slice."""
    elem = 4 if spec['dtype'] == 'float32' else 2
    lens = [int(x) for x in lens]
    dim, bs = spec['head_dim'], spec['block_size']
    b = len(lens)
    kv = sum(2 * kv_heads * length * dim * elem for length in lens)
    qo = b * q_heads * dim * 2 * elem
    idx = sum(-(-length // bs) for length in lens) * 4
    attention = kv + qo + idx + 4 * b
    append = 4 * b * kv_heads * dim * elem
    return attention + append, attention


# ------------------------------------------------------------------ clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ('clocks.sm', 'clocks.max.sm', 'power.draw', 'utilization.gpu',
              'clocks_event_reasons.hw_slowdown', 'clocks_event_reasons.hw_thermal_slowdown',
              'clocks_event_reasons.sw_thermal_slowdown', 'clocks_event_reasons.sw_power_cap')

    def __init__(self, device_index, interval_ms=50):
        self.device_index = device_index
        self.interval_ms = interval_ms
        self.proc = None
        self.file = None

    def __enter__(self):
        self.file = tempfile.NamedTemporaryFile('w+', suffix='.csv', delete=False)
        try:
            self.proc = subprocess.Popen(
                ['nvidia-smi', f'--query-gpu={",".join(self.FIELDS)}', '--format=csv,noheader,nounits',
                 '-i', str(self.device_index), '-lms', str(self.interval_ms)],
                stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        self.file.close()

    def summary(self):
        rows = []
        try:
            for line in Path(self.file.name).read_text().splitlines():
                parts = [p.strip() for p in line.split(',')]
                if len(parts) == len(self.FIELDS):
                    rows.append(parts)
        finally:
            os.unlink(self.file.name)
        if not rows:
            return {'sm_mhz': None, 'sm_max_mhz': None, 'reasons': ['unsampled'], 'samples': 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        loaded = [r for r in rows if (num(r[3]) or 0) >= 50] or rows
        sm = [num(r[0]) for r in loaded if num(r[0]) is not None]
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        reasons = sorted({name for r in loaded for name, flag in zip(names, r[4:8])
                          if flag.lower() == 'active'})
        return {'sm_mhz': statistics.median(sm) if sm else None,
                'sm_max_mhz': num(rows[0][1]),
                'reasons': reasons, 'samples': len(loaded),
                'power_w_max': max((num(r[2]) or 0) for r in rows)}


# ------------------------------------------------------------ CPU baseline

REFERENCE_DIR = ROOT / 'baseline' / '_ref'
CPU_SAMPLE_BYTES = 1 << 30      # fp32 K/V pages of a host sample, at most


def reference_modules():
    """micro-vllm's own ``PagedKVCache`` and ``causal_attention`` from baseline/_ref, or None."""
    if not (REFERENCE_DIR / 'micro_vllm' / '__init__.py').is_file():
        return None
    if str(REFERENCE_DIR) not in sys.path:
        sys.path.append(str(REFERENCE_DIR))
    from micro_vllm.attention import causal_attention
    from micro_vllm.paged_kv_cache import PagedKVCache
    return PagedKVCache, causal_attention


def host_threads():
    """Use every host thread this process may run on; returns the count."""
    import torch
    threads = len(os.sched_getaffinity(0)) if hasattr(os, 'sched_getaffinity') else os.cpu_count()
    torch.set_num_threads(threads)
    return torch.get_num_threads()


def cpu_model():
    try:
        for line in Path('/proc/cpuinfo').read_text().splitlines():
            if line.startswith('model name'):
                return line.split(':', 1)[1].strip()
    except OSError:
        pass
    return 'unknown'


def sample_size(spec, lens, wanted):
    """How many leading sequences fit ``CPU_SAMPLE_BYTES`` of fp32 K/V pages (at least 1)."""
    bs, hkv, dim = spec['block_size'], spec['kv_heads'], spec['head_dim']
    total, count = 0, 0
    for length in lens[:wanted]:
        total += 2 * (-(-int(length) // bs)) * hkv * bs * dim * 4
        if count and total > CPU_SAMPLE_BYTES:
            break
        count += 1
    return count


def host_sample(spec, data, sequences):
    """Host copy of the first ``sequences`` sequences of the workload (their pages only).

    One compact fp32 pool per K and V holds just those sequences' pages (bf16
    widened: the reference's CPU path is timed in fp32), with the block table
    remapped onto it; q and the new K/V rows in fp32. torch CPU tensors.
    """
    import torch

    sample = min(sequences, data['q'].shape[0])
    lens = [int(x) for x in data['host_lens'][:sample].tolist()]
    table = data['host_table'][:sample]
    bs = spec['block_size']
    used = sorted({int(p) for b in range(sample) for p in table[b, :-(-lens[b] // bs)].tolist()})
    remap = {p: i for i, p in enumerate(used)}
    local_table = torch.full_like(table, -1)
    for b in range(sample):
        for j in range(-(-lens[b] // bs)):
            local_table[b, j] = remap[int(table[b, j])]
    idx = torch.tensor(used, device=data['k_pool'].device)
    return dict(
        lens=lens, table=local_table, batch=data['q'].shape[0],
        k_pool=data['k_pool'].index_select(0, idx).float().cpu(),
        v_pool=data['v_pool'].index_select(0, idx).float().cpu(),
        q=data['q'][:sample].float().cpu(),
        k_new=data['k_new'][:sample].float().cpu(),
        v_new=data['v_new'][:sample].float().cpu())


class ReferenceCPUStep:
    """One decode step of micro-vllm's own CPU path over a host sample of the workload.

    Every sequence gets the reference's ``PagedKVCache`` over the sample's one
    shared pool per K and V (its dataclass constructor accepts external pools)
    with its own table row, built once. A step is, per sequence, the per-layer
    work of micro-vllm's model for a paged cache on the CPU (model.py:215-216,
    180-182): ``PagedKVCache.append(0, k_new, v_new)`` (its ``_append_cpu``,
    paged_kv_cache.py:151-176), ``gather(0)`` (:178-193), then
    ``causal_attention(q, k, v, past_length=L-1)`` (attention.py:57-94). Each
    step first rewinds every cache's length to L-1, so the step rewrites the
    same slot with the same row, as a decode step at that position would.
    """

    kind = 'reference'

    def __init__(self, spec, sample, modules):
        import torch

        PagedKVCache, self.causal_attention = modules
        bs = spec['block_size']
        self.sample = sample
        self.caches = []
        for b, length in enumerate(sample['lens']):
            ids = tuple(int(p) for p in sample['table'][b, :-(-length // bs)].tolist())
            self.caches.append(PagedKVCache((sample['k_pool'],), (sample['v_pool'],), [length - 1], ids,
                                            torch.tensor(ids, dtype=torch.int64)))
        hq, dim = sample['q'].shape[1:]
        self.queries = [sample['q'][b].view(1, hq, 1, dim) for b in range(len(sample['lens']))]
        self.keys = [sample['k_new'][b:b + 1] for b in range(len(sample['lens']))]
        self.values = [sample['v_new'][b:b + 1] for b in range(len(sample['lens']))]

    def __call__(self):
        for cache, length, q, key, value in zip(self.caches, self.sample['lens'], self.queries, self.keys,
                                                self.values):
            cache._lengths[0] = length - 1
            cache.append(0, key, value)
            k, v = cache.gather(0)
            self.causal_attention(q, k, v, past_length=length - 1)

    def describe(self, runs, elapsed):
        lens = self.sample['lens']
        return (f'{len(lens)} of {self.sample["batch"]} sequences (lens {min(lens)}..{max(lens)}): micro-vllm\'s '
                f'own PagedKVCache.append (_append_cpu) + gather + causal_attention per sequence, torch fp32 '
                f'(bf16 inputs widened), {runs} steps in {elapsed:.1f} s')


class PortCPUStep:
    """Fallback when micro-vllm is not installed: the oracle's numpy restatement of the same path."""

    kind = 'port'

    def __init__(self, spec, sample):
        self.spec = spec
        self.sample = dict(sample)
        for key in ('k_pool', 'v_pool', 'q', 'k_new', 'v_new', 'table'):
            self.sample[key] = sample[key].numpy()
        self.sample['lens'] = __import__('numpy').asarray(sample['lens'])

    def __call__(self):
        import numpy as np

        from oracle import append_tokens, decode_float

        s = self.sample
        append_tokens(s['k_pool'], s['v_pool'], s['k_new'], s['v_new'], s['table'], s['lens'] - 1)
        decode_float(s['q'], s['k_pool'], s['v_pool'], s['table'], s['lens'], self.spec['head_dim'] ** -0.5,
                     'float32', accum=np.float32)

    def describe(self, runs, elapsed):
        lens = self.sample['lens'].tolist()
        return (f'{len(lens)} of {self.sample["batch"]} sequences (lens {min(lens)}..{max(lens)}): the oracle\'s '
                f'numpy fp32 restatement of micro-vllm\'s CPU path (micro-vllm not installed in baseline/_ref), '
                f'{runs} steps in {elapsed:.1f} s')


def cpu_step(spec, data, sequences):
    """The reference's CPU step over the first ``sequences`` sequences (port if not installed)."""
    sample = host_sample(spec, data, sequences)
    modules = reference_modules()
    return ReferenceCPUStep(spec, sample, modules) if modules else PortCPUStep(spec, sample)


def cpu_record(step, value, runs, elapsed, threads):
    return {'value': value, 'unit': 'GB/s', 'cores': threads, 'kind': step.kind,
            'sample': step.describe(runs, elapsed),
            'host': f'{cpu_model()}, os.cpu_count() {os.cpu_count()}, torch threads {threads}'}


def cpu_baseline(spec, data, q_heads, kv_heads, seconds):
    """Time the reference's CPU path on a sample of this workload for about ``seconds``;
    GB/s on the same algorithmic-bytes basis as the GPU number."""
    threads = host_threads()
    step = cpu_step(spec, data, sample_size(spec, data['host_lens'].tolist(), data['q'].shape[0]))
    nbytes, _ = step_bytes(spec, step.sample['lens'], q_heads, kv_heads)
    step()                                  # first touch of the sample's pages
    runs = 0
    start = time.perf_counter()
    while True:
        step()
        runs += 1
        elapsed = time.perf_counter() - start
        if elapsed >= seconds:
            break
    return cpu_record(step, round(nbytes * runs / elapsed / 1e9, 3), runs, elapsed, threads)


# ------------------------------------------------------------------- ours

def run_ours(args):
    import torch
    import torch.distributed as dist

    from micro_vllm_b200 import cuda_attention, cuda_paged_cache

    rank, world, local_rank = init_distributed(args)
    device = torch.device('cuda', local_rank)
    torch.cuda.set_device(device)
    spec = WORKLOADS[args.workload]
    q_heads, kv_heads, batch_slice = local_geometry(spec, rank, world, args.scaling)
    # Every rank draws the same lengths and page tables (the same shape of work);
    # weak-scaled ranks fill them with their own values.
    value_seed = spec['seed'] + 1 + (rank * 7919 if args.scaling == 'weak' else 0)
    data = make_workload(spec, q_heads, kv_heads, batch_slice, spec['seed'], device, value_seed=value_seed)
    lens_host = data['host_lens'].tolist()
    max_len = max(lens_host)
    step_total, attn_bytes = step_bytes(spec, lens_host, q_heads, kv_heads)
    out = torch.empty_like(data['q'])
    pps = args.pages_per_split

    def separate_step():
        cuda_paged_cache.write_paged_kv(data['k_new'], data['v_new'], data['k_pool'], data['v_pool'],
                                        data['block_table'], positions=data['context_lens'],
                                        positions_are_end=True)
        cuda_attention.paged_decode_attention(data['q'], data['k_pool'], data['v_pool'],
                                              data['block_table'], data['context_lens'],
                                              max_context_len=max_len, out=out,
                                              pages_per_split=pps)

    def fused_step():
        cuda_attention.paged_decode_with_append(data['q'], data['k_new'][:, :, 0], data['v_new'][:, :, 0],
                                                data['k_pool'], data['v_pool'], data['block_table'],
                                                data['context_lens'], max_context_len=max_len, out=out,
                                                pages_per_split=pps)

    step, other_step = (fused_step, separate_step) if args.step == 'fused' else (separate_step, fused_step)

    # The same step with q and the new K rotated (RoPE) inside the decode kernel.
    from micro_vllm_b200.rope import rope_tables
    tables = rope_tables(max_len, data['q'].shape[-1], 1e6, dtype=data['dtype'], device=device)

    def rope_step():
        cuda_attention.paged_decode_with_append(data['q'], data['k_new'][:, :, 0], data['v_new'][:, :, 0],
                                                data['k_pool'], data['v_pool'], data['block_table'],
                                                data['context_lens'], max_context_len=max_len, out=out,
                                                pages_per_split=pps, rope=tables)

    # The same step with the split grid's per-page math on CUDA cores (fp32 FMA)
    # instead of the tensor-core tile: the comparison behind the tensor-core choice.
    def cuda_core_step():
        cuda_attention.paged_decode_with_append(data['q'], data['k_new'][:, :, 0], data['v_new'][:, :, 0],
                                                data['k_pool'], data['v_pool'], data['block_table'],
                                                data['context_lens'], max_context_len=max_len, out=out,
                                                pages_per_split=pps, cuda_core_math=True)

    # The same one-call step on the per-warp stream schedule (one CTA per SM,
    # every warp streaming work items from a queue): the comparison behind
    # keeping the split grid as the default.
    def stream_step():
        cuda_attention.paged_decode_with_append(data['q'], data['k_new'][:, :, 0], data['v_new'][:, :, 0],
                                                data['k_pool'], data['v_pool'], data['block_table'],
                                                data['context_lens'], max_context_len=max_len, out=out,
                                                pages_per_split=pps, schedule='stream')

    try:
        cuda_attention.paged_decode_plan(q_heads, data['k_pool'], max_len, batch=len(lens_host),
                                         pages_per_split=pps, schedule='stream')
        stream_ok = True
    except RuntimeError:
        stream_ok = False

    path, chosen_pps, splits = cuda_attention.paged_decode_plan(
        q_heads, data['k_pool'], max_len, batch=len(lens_host), pages_per_split=pps)
    # The fused step is one decode launch (+ merge); the separate one adds the append kernel.
    launches_per_step = (1 if args.step == 'fused' and path in ('tma_mma', 'tma_mma_stream') else 2) + \
        (1 if splits > 1 else 0)

    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for _ in range(3):
            step()
            other_step()
            rope_step()
            cuda_core_step()
            if stream_ok:
                stream_step()
    torch.cuda.synchronize(device)
    step_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(step_graph, stream=stream):
        step()
    other_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(other_graph, stream=stream):
        other_step()
    rope_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(rope_graph, stream=stream):
        rope_step()
    cuda_core_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(cuda_core_graph, stream=stream):
        cuda_core_step()
    stream_graph = torch.cuda.CUDAGraph() if stream_ok else None
    if stream_ok:
        with torch.cuda.graph(stream_graph, stream=stream):
            stream_step()
    # The step's kernels back to back, KERNEL_CALLS per graph, so their average
    # launch duration excludes the per-replay graph launch gap (roofline).
    kernel_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(kernel_graph, stream=stream):
        for _ in range(KERNEL_CALLS):
            step()
    torch.cuda.synchronize(device)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    visible = os.environ.get('CUDA_VISIBLE_DEVICES')
    smi_index = visible.split(',')[local_rank] if visible else str(local_rank)
    with ClockSampler(smi_index) as clocks:
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step_graph.replay()
            kernel_graph.replay()
        torch.cuda.synchronize(device)
        barrier()
        torch.cuda.synchronize(device)
        # K steps as replays of the graph of KERNEL_CALLS back-to-back steps (the rest,
        # K mod KERNEL_CALLS, as single-step replays): a serving loop replays one graph
        # per decode step of all layers, not one per attention call.
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(args.steps // KERNEL_CALLS):
                kernel_graph.replay()
            for _ in range(args.steps % KERNEL_CALLS):
                step_graph.replay()
            end.record(stream)
        torch.cuda.synchronize(device)
        barrier()
        elapsed_ms = start.elapsed_time(end)

        # The same steps one graph replay each: every step then also pays a graph launch.
        single_reps = min(args.steps, 1000)
        s_start, s_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            s_start.record(stream)
            for _ in range(single_reps):
                step_graph.replay()
            s_end.record(stream)
        torch.cuda.synchronize(device)
        barrier()
        single_ms = s_start.elapsed_time(s_end) / single_reps

        # The step's kernels alone (decode + split merge, and the append kernel in the
        # separate form), average launch duration over back-to-back calls, for the roofline.
        with torch.cuda.stream(stream):
            for _ in range(max(1, args.warmup // KERNEL_CALLS)):
                kernel_graph.replay()
        torch.cuda.synchronize(device)
        reps = max(1, min(args.steps, 2000) // KERNEL_CALLS)
        k_start, k_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            k_start.record(stream)
            for _ in range(reps):
                kernel_graph.replay()
            k_end.record(stream)
        torch.cuda.synchronize(device)
        attn_ms = k_start.elapsed_time(k_end) / (reps * KERNEL_CALLS)

        # The other forms of the step, same loop, reported beside the headline.
        other_reps = min(args.steps, 1000)

        def time_form(graph):
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    graph.replay()
            torch.cuda.synchronize(device)
            barrier()
            torch.cuda.synchronize(device)
            f_start, f_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                f_start.record(stream)
                for _ in range(other_reps):
                    graph.replay()
                f_end.record(stream)
            torch.cuda.synchronize(device)
            barrier()
            return f_start.elapsed_time(f_end) * args.steps / other_reps

        other_ms = time_form(other_graph)
        rope_ms = time_form(rope_graph)
        cuda_core_ms = time_form(cuda_core_graph)
        stream_ms = time_form(stream_graph) if stream_ok else 0.0

        # Rank 0's step alone on the same machine (the other ranks wait at a
        # barrier), timed as the headline is (graphs of KERNEL_CALLS steps):
        # separates what running N GPUs at once costs each GPU from differences
        # between machines.
        solo_ms = 0.0
        if world > 1:
            if rank == 0:
                reps = max(1, min(args.steps, 1000) // KERNEL_CALLS)
                s_start, s_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                with torch.cuda.stream(stream):
                    for _ in range(max(args.warmup // KERNEL_CALLS, 3)):
                        kernel_graph.replay()
                    s_start.record(stream)
                    for _ in range(reps):
                        kernel_graph.replay()
                    s_end.record(stream)
                torch.cuda.synchronize(device)
                solo_ms = s_start.elapsed_time(s_end) / (reps * KERNEL_CALLS)
            barrier()

        # End to end through the public API: pinned host inputs in, output back out.
        e2e = run_e2e(args, data, max_len, pps, stream, device, barrier)
    clock_summary = clocks.summary()
    del step_graph, kernel_graph, other_graph, rope_graph, cuda_core_graph, stream_graph
    rank_us_per_launch = per_rank_values(attn_ms * 1e3, rank, world, device)
    rank_separate_us = per_rank_values(other_ms / args.steps * 1e3, rank, world, device)
    strong = None
    if args.workload == DEFAULT_WORKLOAD and not args.pages_per_split and not args.no_strong_scaling:
        strong = strong_scaling(rank, world, device, barrier)

    times = torch.tensor([elapsed_ms, attn_ms, e2e['ms'], other_ms, rope_ms, cuda_core_ms, stream_ms, single_ms,
                          e2e['each_ms']],
                         dtype=torch.float64, device=device)
    totals = torch.tensor([float(step_total), float(attn_bytes)], dtype=torch.float64, device=device)
    rank_ms_per_step = per_rank_values(elapsed_ms / args.steps, rank, world, device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        dist.all_reduce(totals, op=dist.ReduceOp.SUM)
    elapsed_ms, attn_ms, e2e_ms, other_ms, rope_ms, cuda_core_ms, stream_ms, single_ms, e2e_each_ms = times.tolist()
    job_step_bytes, job_attn_bytes = totals.tolist()
    ms_per_step = elapsed_ms / args.steps
    value = job_step_bytes * args.steps / (elapsed_ms / 1e3) / 1e9
    e2e_value = job_step_bytes * args.steps / (e2e_ms / 1e3) / 1e9

    result = None
    if rank == 0:
        peak, peak_kind = peak_hbm()
        achieved = step_total / (attn_ms / 1e3) / 1e9
        # The capture is of the default step form on one GPU's config-sized slice.
        traffic = (NCU_TRAFFIC_BYTES.get((args.workload, path))
                   if args.step == 'fused' and not args.pages_per_split
                   and (world == 1 or args.scaling == 'weak') else None)
        batch = len(lens_host)
        result = {
            'metric': METRIC,
            'value': round(value, 1),
            'unit': 'GB/s',
            'n_gpus': world,
            'steps': args.steps,
            'warmup': args.warmup,
            'ms_per_step': round(ms_per_step, 6),
            'higher_is_better': True,
            'scaling': args.scaling if world > 1 else 'weak',
            'vs_baseline': None,
            'dtype': {'bfloat16': 'bf16', 'float16': 'fp16', 'float32': 'fp32'}[spec['dtype']],
            'data': 'synthetic (seeded, on device)',
            'config': {
                'workload': (f'{args.workload}: paged GQA decode layer, batch {spec["batch"]}, '
                             f'{spec["q_heads"]} q / {spec["kv_heads"]} kv heads, head_dim '
                             f'{spec["head_dim"]}, block {spec["block_size"]}, lens {spec["lens"]}'),
                'per_rank': {'batch': batch, 'q_heads': q_heads, 'kv_heads': kv_heads},
                'step': ('append 1 token/sequence + paged decode attention (1 layer), '
                         + ('one call: paged_decode_with_append' if args.step == 'fused' else
                            'two calls: write_paged_kv + paged_decode_attention')),
                'l2': f'inputs larger than L2: KV pool {2 * data["k_pool"].numel() * data["k_pool"].element_size() / 1e9:.2f} GB per GPU',
                'parallelism': f'kv-head sharded x{world}, {args.scaling}' if world > 1 else 'single GPU',
                'timing': (f'CUDA events around K steps run as replays of a CUDA graph of {KERNEL_CALLS} back-to-back '
                           'steps (a serving loop replays one graph per decode step of all layers), max over ranks'),
                'kernel_path': path, 'pages_per_split': chosen_pps, 'max_splits': splits,
            },
            'us_per_layer': round(ms_per_step * 1e3, 3),
            'ms_per_step_single_replay': round(single_ms, 6),
            'decode_tokens_per_s': round(spec['batch'] / (ms_per_step / 1e3), 1),
            'pct_of_hbm_peak': round(100 * value / world / peak, 2),
            'roofline': {
                'bound': 'hbm',
                'kernel': (STEP_KERNELS.get(path, path) if args.step == 'fused' else
                           'write_paged_kv_kernel + ' + STEP_KERNELS.get(path, path).replace(' (append fused)', '')),
                'timing': (f'CUDA events around graphs of {KERNEL_CALLS} back-to-back steps: '
                           'average launch duration without the per-replay graph launch gap'),
                'achieved': round(achieved, 1),
                'peak': peak,
                'peak_kind': f'{peak_kind} copy bandwidth (MEASURED_PEAKS.json hbm_gbs)'
                             if peak_kind == 'measured' else 'fallback 6.65 TB/s',
                'unit': 'GB/s',
                'frac': round(achieved / peak, 4),
                'us_per_launch': round(attn_ms * 1e3, 3),
                'algorithmic_bytes_per_launch': step_total,
                'traffic': traffic,
                'traffic_source': TRAFFIC_SOURCES.get(path) if traffic else None,
            },
            'e2e': {'value': round(e2e_value, 1), 'unit': 'GB/s',
                    'h2d_bytes_per_step': e2e['h2d'], 'd2h_bytes_per_step': e2e['d2h'],
                    'us_per_step': round(e2e_ms / args.steps * 1e3, 3),
                    'us_per_step_issued_one_by_one': round(e2e_each_ms * 1e3, 3),
                    'how': ('public API (PagedDecodeStep) per step: packed q/k/v + lengths uploaded from '
                            'pinned host memory and the output downloaded to pinned host memory, on '
                            f'their own streams; issued in blocks of {KERNEL_CALLS} steps (the uploads of '
                            'a block while the previous block computes, its calls back to back, then its '
                            'downloads; 2 blocks of buffer slots). us_per_step_issued_one_by_one: each '
                            'step waits for its own upload and two slots')},
            'step_forms_us': {args.step: round(ms_per_step * 1e3, 3),
                              ('separate' if args.step == 'fused' else 'fused'):
                                  round(other_ms / args.steps * 1e3, 3),
                              'fused_with_rope': round(rope_ms / args.steps * 1e3, 3),
                              'fused_cuda_core_math': round(cuda_core_ms / args.steps * 1e3, 3),
                              'fused_stream_schedule': round(stream_ms / args.steps * 1e3, 3) if stream_ok else None},
            'clocks': clock_summary,
            'gpu_launches': launches_per_step * args.steps,
        }
        if world > 1:
            # ms_per_step is the slowest of these; the kernels' own times per rank beside them.
            result['per_rank_ms_per_step'] = [round(t, 6) for t in rank_ms_per_step]
            result['per_rank_us_per_launch'] = [round(t, 3) for t in rank_us_per_launch]
            result['per_rank_separate_step_us'] = [round(t, 3) for t in rank_separate_us]
            result['rank0_alone_ms_per_step'] = round(solo_ms, 6)
        if strong is not None:
            result['strong_scaling'] = strong
        if world == 1 and not args.no_cpu_baseline:
            result['cpu_baseline'] = cpu_baseline(spec, data, q_heads, kv_heads, args.cpu_seconds)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()
    return result


STRONG_WORKLOADS = ('qwen3_8b_long_bf16', 'qwen72b_bf16')
STRONG_REPLAYS = 40


def time_one_call_step(data, stream, device, replays):
    """Device time (ms) of one replay of a CUDA graph holding the one-call step on ``data``."""
    import torch

    from micro_vllm_b200 import cuda_attention

    max_len = int(data['host_lens'].max())
    out = torch.empty_like(data['q'])

    def step():
        cuda_attention.paged_decode_with_append(data['q'], data['k_new'][:, :, 0], data['v_new'][:, :, 0],
                                                data['k_pool'], data['v_pool'], data['block_table'],
                                                data['context_lens'], max_context_len=max_len, out=out)

    stream.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(stream):
        for _ in range(3):
            step()
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(3):
            graph.replay()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(replays):
            graph.replay()
        end.record(stream)
    torch.cuda.synchronize(device)
    del graph
    return start.elapsed_time(end) / replays


def strong_scaling(rank, world, device, barrier):
    """The long-context (Qwen3-8B geometry) and batch-256 (Qwen2.5-72B geometry)
    layers split over the ranks by KV head -- one KV head per GPU at 8 -- each rank
    timing the one-call step on its shard (CUDA-graph replays, max over ranks),
    plus the whole layer on rank 0's GPU alone in the same run for comparison.
    Every rank takes the same collective steps in the same order."""
    import torch

    from micro_vllm_b200 import cuda_attention

    stream = torch.cuda.Stream(device)
    records = {}
    for name in STRONG_WORKLOADS:
        spec = WORKLOADS[name]
        q_heads, kv_heads, batch_slice = local_geometry(spec, rank, world, 'strong')
        data = make_workload(spec, q_heads, kv_heads, batch_slice, spec['seed'], device)
        lens = data['host_lens'].tolist()
        plan = cuda_attention.paged_decode_plan(q_heads, data['k_pool'], max(lens), batch=len(lens))
        nbytes, _ = step_bytes(spec, lens, q_heads, kv_heads)
        barrier()
        ms = time_one_call_step(data, stream, device, STRONG_REPLAYS)
        barrier()
        del data
        per_rank_us = per_rank_values(ms * 1e3, rank, world, device)
        per_rank_bytes = per_rank_values(float(nbytes), rank, world, device)
        one_gpu_us = per_rank_us[0]
        if world > 1:
            if rank == 0:
                whole = make_workload(spec, spec['q_heads'], spec['kv_heads'], (0, spec['batch']), spec['seed'],
                                      device)
                one_gpu_us = time_one_call_step(whole, stream, device, STRONG_REPLAYS) * 1e3
                del whole
            barrier()
        torch.cuda.empty_cache()
        slowest = max(per_rank_us)
        total = sum(per_rank_bytes)
        records[name] = {
            'workload': (f'{name}: batch {spec["batch"]}, {spec["q_heads"]} q / {spec["kv_heads"]} kv heads, '
                         f'head_dim {spec["head_dim"]}, lens {spec["lens"]}'),
            'per_rank': {'batch': len(lens), 'q_heads': q_heads, 'kv_heads': kv_heads, 'plan': list(plan)},
            'us_per_layer': round(slowest, 3),
            'per_rank_us': [round(t, 3) for t in per_rank_us],
            'aggregate_gbs': round(total / (slowest * 1e3), 1),
            'per_gpu_gbs': round(total / (slowest * 1e3) / world, 1),
            'us_per_layer_one_gpu': round(one_gpu_us, 3),
            'speedup_vs_one_gpu': round(one_gpu_us / slowest, 3),
            'strong_efficiency': round(one_gpu_us / (slowest * world), 3),
            'timing': (f'one-call step (append + decode), CUDA events around {STRONG_REPLAYS} graph replays per '
                       'rank, max over ranks; one-GPU time: the whole layer on rank 0 in the same run'),
        }
    return records


def run_e2e(args, data, max_len, pps, stream, device, barrier):
    """Same step through the public API with host inputs and a host result.

    Every step uploads its inputs from pinned host memory in one copy -- q and
    the new K/V rows packed as one [B, Hq + 2 Hkv, D] block (the layout of a
    fused QKV projection) followed by the lengths -- runs the step through a bound
    ``PagedDecodeStep`` (or the two-call form), and downloads its output into
    pinned host memory. Uploads and downloads run on their own streams. The
    reported figure issues the steps in blocks of KERNEL_CALLS (the block's
    uploads while the previous block computes, its calls back to back, then its
    downloads), so consecutive steps' kernels overlap as in the device timing;
    the steps issued one by one (each waiting for its own upload, two buffer
    slots) are timed too, since an event wait between two steps' kernels keeps
    the next decode from launching early.
    """
    import torch

    from micro_vllm_b200 import cuda_attention, cuda_paged_cache

    batch, hq, dim = data['q'].shape
    hkv = data['k_new'].shape[1]
    slots = 2
    # One upload per step: the packed q/k/v rows, then the int32 lengths, as raw bytes.
    packed = torch.cat([data['q'], data['k_new'][:, :, 0], data['v_new'][:, :, 0]], dim=1)
    qkv_bytes = packed.numel() * packed.element_size()
    lens_bytes = data['context_lens'].numel() * data['context_lens'].element_size()
    staging = torch.cat([packed.reshape(-1).view(torch.uint8), data['context_lens'].view(torch.uint8)])
    host_in = [staging.cpu().pin_memory() for _ in range(slots)]
    dev_in = [torch.empty_like(staging) for _ in range(slots)]
    dev_qkv = [buf[:qkv_bytes].view(packed.dtype).view(packed.shape) for buf in dev_in]
    dev_lens = [buf[qkv_bytes:].view(data['context_lens'].dtype) for buf in dev_in]
    dev_out = [torch.empty_like(data['q']) for _ in range(slots)]
    host_out = [torch.empty(data['q'].shape, dtype=data['q'].dtype).pin_memory() for _ in range(slots)]
    h2d = qkv_bytes + lens_bytes
    d2h = host_out[0].numel() * host_out[0].element_size()
    views = [(qkv[:, :hq], qkv[:, hq:hq + hkv], qkv[:, hq + hkv:]) for qkv in dev_qkv]
    bound = cuda_attention.PagedDecodeStep(data['k_pool'], data['v_pool'], data['block_table'],
                                           num_q_heads=hq, max_context_len=max_len, pages_per_split=pps)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    loaded = [torch.cuda.Event() for _ in range(slots)]
    computed = [torch.cuda.Event() for _ in range(slots)]
    read = [torch.cuda.Event() for _ in range(slots)]
    for event in computed + read:
        event.record(stream)

    def step(i):
        s = i % slots
        up.wait_event(computed[s])          # step i-2 has consumed this slot's inputs
        with torch.cuda.stream(up):
            dev_in[s].copy_(host_in[s], non_blocking=True)
        loaded[s].record(up)
        stream.wait_event(loaded[s])
        stream.wait_event(read[s])          # step i-2's output has been downloaded
        q, key, value = views[s]
        with torch.cuda.stream(stream):
            if args.step == 'fused':
                bound(q, dev_lens[s], dev_out[s], key=key, value=value)
            else:
                cuda_paged_cache.write_paged_kv(key.unsqueeze(2), value.unsqueeze(2), data['k_pool'],
                                                data['v_pool'], data['block_table'], positions=dev_lens[s],
                                                positions_are_end=True)
                bound(q, dev_lens[s], dev_out[s])
        computed[s].record(stream)
        down.wait_event(computed[s])
        with torch.cuda.stream(down):
            host_out[s].copy_(dev_out[s], non_blocking=True)
        read[s].record(down)

    steps = min(args.steps, 1000)
    for i in range(max(args.warmup, 3)):
        step(i)
    torch.cuda.synchronize(device)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    up.wait_event(start)
    for i in range(steps):
        step(i)
    stream.wait_stream(up)
    stream.wait_stream(down)
    end.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    each_ms = start.elapsed_time(end) / steps

    # The same per-step copies and calls issued in blocks of KERNEL_CALLS steps
    # (the grouping of the device timing): the block's uploads (one per step,
    # 2 x KERNEL_CALLS buffer slots) on the upload stream while the previous
    # block computes, its steps' calls back to back on the compute stream with
    # no event between them (so each decode launches early and overlaps the
    # previous merge), then one download per step.
    block = KERNEL_CALLS
    b_host_in = [staging.cpu().pin_memory() for _ in range(2 * block)]
    b_dev_in = [torch.empty_like(staging) for _ in range(2 * block)]
    b_qkv = [buf[:qkv_bytes].view(packed.dtype).view(packed.shape) for buf in b_dev_in]
    b_lens = [buf[qkv_bytes:].view(data['context_lens'].dtype) for buf in b_dev_in]
    b_views = [(qkv[:, :hq], qkv[:, hq:hq + hkv], qkv[:, hq + hkv:]) for qkv in b_qkv]
    b_dev_out = [torch.empty_like(data['q']) for _ in range(2 * block)]
    b_host_out = [torch.empty(data['q'].shape, dtype=data['q'].dtype).pin_memory() for _ in range(2 * block)]
    b_loaded = [torch.cuda.Event() for _ in range(2)]
    b_computed = [torch.cuda.Event() for _ in range(2)]
    b_read = [torch.cuda.Event() for _ in range(2)]
    for event in b_computed + b_read:
        event.record(stream)

    def run_block(j):
        half = j % 2
        slots_j = range(half * block, half * block + block)
        up.wait_event(b_computed[half])      # block j-2 has consumed these input slots
        with torch.cuda.stream(up):
            for s in slots_j:
                b_dev_in[s].copy_(b_host_in[s], non_blocking=True)
        b_loaded[half].record(up)
        stream.wait_event(b_loaded[half])
        stream.wait_event(b_read[half])      # block j-2's outputs have been downloaded
        with torch.cuda.stream(stream):
            for s in slots_j:
                q, key, value = b_views[s]
                if args.step == 'fused':
                    bound(q, b_lens[s], b_dev_out[s], key=key, value=value)
                else:
                    cuda_paged_cache.write_paged_kv(key.unsqueeze(2), value.unsqueeze(2), data['k_pool'],
                                                    data['v_pool'], data['block_table'], positions=b_lens[s],
                                                    positions_are_end=True)
                    bound(q, b_lens[s], b_dev_out[s])
        b_computed[half].record(stream)
        down.wait_event(b_computed[half])
        with torch.cuda.stream(down):
            for s in slots_j:
                b_host_out[s].copy_(b_dev_out[s], non_blocking=True)
        b_read[half].record(down)

    blocks = max(1, steps // block)
    for j in range(3):
        run_block(j)
    torch.cuda.synchronize(device)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    up.wait_event(start)
    for j in range(blocks):
        run_block(j)
    stream.wait_stream(up)
    stream.wait_stream(down)
    end.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    block_ms = start.elapsed_time(end) / (blocks * block)
    # Scale to the main loop's step count so value and e2e share one unit basis.
    return {'ms': block_ms * args.steps, 'each_ms': each_ms, 'h2d': h2d, 'd2h': d2h}


# -------------------------------------------------------------- reference

def run_reference(args):
    """The reference's CPU path (micro-vllm's own code from baseline/_ref) on this host's cores.

    Each step is one pass of ``ReferenceCPUStep`` over a bounded sample of the
    workload: all sequences, or the leading ones when K + W steps would take
    more than ~2 minutes (or their pages more than ``CPU_SAMPLE_BYTES``), timed
    with the wall clock; value is the median GB/s over the K timed steps.
    """
    rank = int(os.environ.get('RANK', '0'))
    if rank != 0:
        return None

    spec = WORKLOADS[args.workload]
    threads = host_threads()
    data = make_workload(spec, spec['q_heads'], spec['kv_heads'], (0, spec['batch']), spec['seed'], 'cpu')
    sequences = sample_size(spec, data['host_lens'].tolist(), spec['batch'])
    budget = 120.0
    while True:
        step = cpu_step(spec, data, sequences)
        step()
        start = time.perf_counter()
        step()
        one = time.perf_counter() - start
        if sequences == 1 or one * (args.steps + args.warmup) <= budget:
            break
        sequences = max(1, int(sequences * budget / (one * (args.steps + args.warmup)) * 0.9))
    nbytes, _ = step_bytes(spec, step.sample['lens'], spec['q_heads'], spec['kv_heads'])
    values = []
    total_elapsed = 0.0
    for i in range(args.warmup + args.steps):
        start = time.perf_counter()
        step()
        elapsed = time.perf_counter() - start
        if i >= args.warmup:
            values.append(nbytes / elapsed / 1e9)
            total_elapsed += elapsed
    value = round(statistics.median(values), 3)
    record = cpu_record(step, value, args.steps, total_elapsed, threads)
    line = {
        'impl': 'reference',
        'metric': METRIC, 'value': value, 'unit': 'GB/s', 'n_gpus': args.gpus,
        'steps': args.steps, 'warmup': args.warmup,
        'ms_per_step': round(total_elapsed / args.steps * 1e3, 6),
        'higher_is_better': True, 'scaling': args.scaling, 'vs_baseline': None,
        'dtype': 'fp32 (bf16 inputs widened)', 'data': 'synthetic (seeded)',
        'config': {'workload': args.workload, 'sample': record['sample']},
        'cpu_baseline': record,
        'e2e': {'value': value, 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0},
    }
    gpu = reference_gpu_kernels(spec)
    if gpu is not None:
        line['reference_gpu_kernels'] = gpu
    return line


def reference_gpu_kernels(spec, steps=5, warmup=2):
    """The reference's own CUDA extensions on the workload, for comparison.

    oracle/build_ref.py compiles them from the reference's sources into
    oracle/_ref. One step is the reference model's decode-step attention for
    every sequence, one request per call as the reference serves them:
    ``write_paged_kv`` of the new K/V row then ``_decode_attention_paged``
    (src/micro_vllm/model.py:215-216, 177). bf16 workloads run in fp16 (the
    same bytes; the reference kernels take fp16/fp32 only). Device time of
    eager steps between CUDA events. None when the modules or a GPU are absent.
    """
    import torch

    from oracle.build_ref import load

    attn, cache = load('_micro_vllm_decode_attention'), load('_micro_vllm_paged_cache')
    if attn is None or cache is None or not torch.cuda.is_available():
        return None
    run_spec = dict(spec, dtype='float16') if spec['dtype'] == 'bfloat16' else dict(spec)
    device = torch.device('cuda', 0)
    try:
        data = make_workload(run_spec, spec['q_heads'], spec['kv_heads'], (0, spec['batch']), spec['seed'], device)
        lens = [int(x) for x in data['host_lens'].tolist()]
        bs = spec['block_size']
        tables = [data['host_table'][b, :-(-n // bs)].to(torch.int64).to(device) for b, n in enumerate(lens)]
        queries = [data['q'][b:b + 1].unsqueeze(2) for b in range(len(lens))]
        keys = [data['k_new'][b:b + 1] for b in range(len(lens))]
        values = [data['v_new'][b:b + 1] for b in range(len(lens))]
        k_pool, v_pool = data['k_pool'], data['v_pool']

        def step():
            for b, n in enumerate(lens):
                cache.write_paged_kv(keys[b], values[b], k_pool, v_pool, tables[b], n - 1)
                attn._decode_attention_paged(queries[b], k_pool, v_pool, tables[b], n)

        for _ in range(warmup):
            step()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            step()
        end.record()
        torch.cuda.synchronize(device)
        ms = start.elapsed_time(end) / steps
    except RuntimeError as exc:
        return {'unavailable': str(exc).splitlines()[0][:200]}
    total, _ = step_bytes(run_spec, lens, spec['q_heads'], spec['kv_heads'])
    return {'value': round(total / (ms * 1e-3) / 1e9, 1), 'unit': 'GB/s', 'us_per_step': round(ms * 1e3, 1),
            'dtype': 'fp16' + (' (bf16 workload: same bytes)' if spec['dtype'] == 'bfloat16' else ''),
            'how': (f'reference CUDA extensions built from its sources (oracle/build_ref.py): per sequence '
                    f'write_paged_kv + _decode_attention_paged, {len(lens)} sequences per step, eager, '
                    f'CUDA events around {steps} steps')}


# ------------------------------------------------------- greedy generation

GENERATE_WORKLOADS = {
    # Qwen2.5-1.5B architecture, random init N(0, 0.02^2) (RMSNorm scales 1), bf16;
    # batch 32 prompts of 512 uniform-random token IDs, 128 new tokens, 16-token pages.
    'qwen15b_generate': dict(num_hidden_layers=28, hidden_size=1536, intermediate_size=8960,
                             num_attention_heads=12, num_key_value_heads=2, vocab_size=151936,
                             max_position_embeddings=32768, rope_theta=1000000.0, rms_norm_eps=1e-6,
                             tie_word_embeddings=True, batch=32, prompt_len=512, new_tokens=128, seed=2024),
}


def _random_qwen2(spec, device, dtype):
    """Random-init weights in the reference's checkpoint naming, generated on the device."""
    import torch
    from types import SimpleNamespace

    gen = torch.Generator(device=device).manual_seed(spec['seed'])
    hidden, inter = spec['hidden_size'], spec['intermediate_size']
    dim = hidden // spec['num_attention_heads']
    kv = spec['num_key_value_heads'] * dim

    def normal(*shape):
        out = torch.empty(shape, dtype=dtype, device=device)
        flat = out.view(-1)
        for start in range(0, flat.numel(), 1 << 26):
            piece = torch.randn(min(1 << 26, flat.numel() - start), generator=gen, device=device)
            flat[start:start + piece.numel()] = piece.mul_(0.02)
        return out

    ones = lambda n: torch.ones(n, dtype=dtype, device=device)  # noqa: E731
    weights = {'model.embed_tokens.weight': normal(spec['vocab_size'], hidden), 'model.norm.weight': ones(hidden)}
    for i in range(spec['num_hidden_layers']):
        p = f'model.layers.{i}.'
        weights.update({
            p + 'input_layernorm.weight': ones(hidden), p + 'post_attention_layernorm.weight': ones(hidden),
            p + 'self_attn.q_proj.weight': normal(hidden, hidden), p + 'self_attn.k_proj.weight': normal(kv, hidden),
            p + 'self_attn.v_proj.weight': normal(kv, hidden), p + 'self_attn.q_proj.bias': normal(hidden),
            p + 'self_attn.k_proj.bias': normal(kv), p + 'self_attn.v_proj.bias': normal(kv),
            p + 'self_attn.o_proj.weight': normal(hidden, hidden),
            p + 'mlp.gate_proj.weight': normal(inter, hidden), p + 'mlp.up_proj.weight': normal(inter, hidden),
            p + 'mlp.down_proj.weight': normal(hidden, inter)})
    keys = ('num_hidden_layers', 'hidden_size', 'intermediate_size', 'num_attention_heads', 'num_key_value_heads',
            'vocab_size', 'max_position_embeddings', 'rope_theta', 'rms_norm_eps', 'tie_word_embeddings')
    config = SimpleNamespace(model_type='qwen2', hidden_act='silu', rope_scaling=None, use_sliding_window=False,
                             layer_types=['full_attention'] * spec['num_hidden_layers'], head_dim=None,
                             partial_rotary_factor=1.0, **{k: spec[k] for k in keys})
    return weights, config


def run_generate(args):
    """Greedy generation of the batched runtime: decode tokens/s and the attention share."""
    import torch

    from micro_vllm_b200.generate import GreedyDecoder
    from micro_vllm_b200.runtime import prepare_model

    if int(os.environ.get('WORLD_SIZE', '1')) > 1 and int(os.environ.get('RANK', '0')) > 0:
        return None  # one replica on rank 0; the other ranks idle
    spec = GENERATE_WORKLOADS[args.workload]
    device = torch.device('cuda', int(os.environ.get('LOCAL_RANK', '0')))
    torch.cuda.set_device(device)
    weights, config = _random_qwen2(spec, device, torch.bfloat16)
    model = prepare_model(weights, config)
    batch, prompt_len, new = spec['batch'], spec['prompt_len'], spec['new_tokens']
    prompts_host = torch.randint(0, spec['vocab_size'], (batch, prompt_len),
                                 generator=torch.Generator().manual_seed(spec['seed']))
    if args.nvtx_steps:
        # Profiling aid: eager prefill and decode steps in named NVTX ranges.
        decoder = GreedyDecoder(model, batch, prompt_len + args.nvtx_steps + 1, use_graph=False)
        prompts = prompts_host.to(device)
        decoder.run(prompts, 2)
        decoder.cache.reset()
        torch.cuda.synchronize(device)
        torch.cuda.nvtx.range_push('prefill')
        decoder.tokens.copy_(model.prefill(prompts, decoder.cache).argmax(dim=-1))
        torch.cuda.synchronize(device)
        torch.cuda.nvtx.range_pop()
        torch.cuda.nvtx.range_push('decode')
        for _ in range(args.nvtx_steps):
            decoder.step()
        torch.cuda.synchronize(device)
        torch.cuda.nvtx.range_pop()
        return None
    decoder = GreedyDecoder(model, batch, prompt_len + new - 1)
    prompts = prompts_host.to(device)
    for _ in range(max(args.warmup, 1)):           # warm-up: cuBLAS plans, graph capture
        decoder.run(prompts, 4)
    torch.cuda.synchronize(device)

    # Prefill and the decode steps, timed on the device.
    with ClockSampler(str(device.index)) as clocks:
        events = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        decoder.cache.reset()
        events[0].record()
        logits = model.prefill(prompts, decoder.cache)
        decoder.tokens.copy_(logits.argmax(dim=-1))
        events[1].record()
        for _ in range(new - 1):
            decoder.step()
        events[2].record()
        torch.cuda.synchronize(device)
        prefill_ms = events[0].elapsed_time(events[1])
        decode_ms = events[1].elapsed_time(events[2])

        # Attention alone: the 28 layers' decode-step calls on the same buffers, as one graph.
        hq, hkv, d = model.num_heads, model.num_kv_heads, model.head_dim
        qkv = torch.randn(batch, hq + 2 * hkv, d, device=device).to(torch.bfloat16)
        lens = decoder.cache.lengths.clone()
        stream = torch.cuda.Stream(device)
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            for step in model._steps:
                step(qkv[:, :hq], lens, key=qkv[:, hq:hq + hkv], value=qkv[:, hq + hkv:])
        torch.cuda.synchronize(device)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for step in model._steps:
                step(qkv[:, :hq], lens, key=qkv[:, hq:hq + hkv], value=qkv[:, hq + hkv:])
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 50
        a0.record()
        for _ in range(reps):
            graph.replay()
        a1.record()
        torch.cuda.synchronize(device)
        attention_ms = a0.elapsed_time(a1) / reps

        # End to end through the public API: pinned host prompts in, host tokens out
        # (a serving loop keeps its GreedyDecoder: cache and captured graph reused).
        pinned = prompts_host.pin_memory()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        tokens = decoder.run(pinned.to(device, non_blocking=True), new).cpu()
        e1.record()
        torch.cuda.synchronize(device)
        e2e_ms = e0.elapsed_time(e1)
        path, _, splits = model._steps[0].plan
    del graph
    step_ms = decode_ms / (new - 1)
    decode_tps = batch * (new - 1) / (decode_ms / 1e3)
    weight_bytes = sum(t.numel() * t.element_size() for t in model.layers[0].values()) * model.num_layers + \
        model.embedding.numel() * model.embedding.element_size()
    peak, peak_kind = peak_hbm()
    return {
        'metric': 'decode tokens/s (greedy generation, batch 32, random-init Qwen2.5-1.5B)',
        'value': round(decode_tps, 1),
        'unit': 'tokens/s',
        'n_gpus': 1,
        'steps': new - 1,
        'warmup': max(args.warmup, 1),
        'ms_per_step': round(step_ms, 4),
        'higher_is_better': True,
        'scaling': 'weak',
        'vs_baseline': None,
        'dtype': 'bf16',
        'data': 'synthetic (random-init weights N(0, 0.02^2), uniform-random prompt token IDs)',
        'config': {'workload': (f'{args.workload}: 28 layers, hidden 1536, 12/2 heads, head_dim 128, '
                                f'FFN 8960, vocab 151936, batch {batch} x {prompt_len} prompt tokens, '
                                f'{new} new tokens, 16-token pages'),
                   'timing': 'CUDA events: prefill, then the 127 graph-replayed decode steps',
                   'attention': 'paged_decode_with_append (RoPE + append + paged decode) per layer'},
        'prefill_ms': round(prefill_ms, 3),
        'attention_share': round(attention_ms / step_ms, 4),
        'attention_ms_per_step': round(attention_ms, 4),
        'weights_gb': round(weight_bytes / 1e9, 3),
        'weight_stream_gbs': round(weight_bytes / (step_ms / 1e3) / 1e9, 1),
        'roofline': {'bound': 'hbm', 'achieved': round(weight_bytes / (step_ms / 1e3) / 1e9, 1), 'peak': peak,
                     'unit': 'GB/s', 'frac': round(weight_bytes / (step_ms / 1e3) / 1e9 / peak, 4),
                     'what': 'decode step: every weight byte read once per step (GEMMs at M = 32)',
                     'peak_kind': peak_kind},
        'e2e': {'value': round(batch * new / (e2e_ms / 1e3), 1), 'unit': 'tokens/s (all new tokens, incl. prefill)',
                'ms': round(e2e_ms, 2), 'h2d_bytes_per_step': prompts_host.numel() * 8,
                'd2h_bytes_per_step': tokens.numel() * 8,
                'how': 'GreedyDecoder.run from pinned host prompts to host tokens, one batch'},
        'decode_path': path,
        'tokens_checksum': int(tokens.sum()),
        'clocks': clocks.summary(),
        # This library's kernels in the timed prefill + decode: RoPE q, RoPE K and the
        # append per prefill layer; the decode kernel (+ split merge) per decode layer.
        'gpu_launches': model.num_layers * (3 + (new - 1) * (2 if splits > 1 else 1)),
    }


def run_kernels(args):
    """Each of this library's kernels on the config-4 shapes, CUDA-event timed (and a
    fixed sequence of calls a profiler can select launches from)."""
    import torch

    from micro_vllm_b200 import cuda_attention
    from micro_vllm_b200.rope import apply_rope, rope_tables
    from micro_vllm_b200.row_ops import rms_norm, silu_mul

    device = torch.device('cuda', int(os.environ.get('LOCAL_RANK', '0')))
    torch.cuda.set_device(device)
    gen = torch.Generator(device=device).manual_seed(5)
    bf16 = torch.bfloat16

    def randn(*shape, dtype=bf16):
        return torch.randn(shape, generator=gen, device=device).to(dtype)

    def pool(batch, kv_heads, dim, lo, hi, dtype, seed):
        lens = torch.randint(lo, hi + 1, (batch,), generator=torch.Generator().manual_seed(seed))
        pages = (lens + 15) // 16
        table = torch.full((batch, int(pages.max())), -1, dtype=torch.int32)
        perm = torch.randperm(int(pages.sum()), generator=torch.Generator().manual_seed(seed + 1)).to(torch.int32)
        offset = 0
        for b, n in enumerate(pages.tolist()):
            table[b, :n] = perm[offset:offset + n]
            offset += n
        k = randn(int(pages.sum()), kv_heads, 16, dim, dtype=dtype)
        v = randn(int(pages.sum()), kv_heads, 16, dim, dtype=dtype)
        return k, v, table.to(device), lens.to(torch.int32).to(device)

    cos, sin = rope_tables(4096, 128, 1e6, dtype=bf16, device=device)
    g_k, g_v, g_table, g_lens = pool(32, 2, 128, 513, 639, bf16, 1)     # config-4 decode attention
    g_q, g_rows = randn(32, 12, 128), randn(32, 2, 2, 128)
    c_k, c_v, c_table, c_lens = pool(4, 2, 64, 1, 512, torch.float32, 2)  # config-1 fp32 decode
    c_q, c_rows = randn(4, 14, 64, dtype=torch.float32), randn(4, 2, 2, 64, dtype=torch.float32)
    x, h, w = randn(32, 12, 512, 128), randn(16384, 1536), torch.ones(1536, dtype=bf16, device=device)
    gate_up = randn(16384, 2 * 8960)
    # Contiguous caches [64, 4, 4096, 128] (Qwen2.5-7B geometry), lengths U[1024, 4096].
    cc_k, cc_v = randn(64, 4, 4096, 128), randn(64, 4, 4096, 128)
    cc_lens = torch.randint(1024, 4097, (64,), generator=torch.Generator().manual_seed(3)).to(torch.int32)
    cc_q = randn(64, 28, 128)
    # Chunks of 4 new tokens per sequence over pages (Qwen2.5-7B geometry, 16 sequences).
    ch_k, ch_v, ch_table, ch_lens = pool(16, 4, 128, 1024, 4096, bf16, 4)
    ch_q = randn(16, 28, 4, 128)
    # A 256-token prefill chunk after 1024 cached tokens (Qwen2.5-1.5B heads, 4 sequences).
    cp_k, cp_v, cp_table, cp_lens = pool(4, 2, 128, 1280, 1280, bf16, 5)
    cp_q = randn(4, 12, 256, 128)
    # Flops of a chunk: each query row attends its causal prefix, 4 D flops per (row, token).
    chunk_flops = lambda lens, tokens, q_heads, dim: sum(  # noqa: E731
        4 * dim * q_heads * (int(n) - t) for n in lens.tolist() for t in range(tokens))
    kv_bytes = lambda lens, heads, dim, elem: int(lens.to(torch.int64).sum()) * 2 * heads * dim * elem  # noqa: E731
    algorithmic = {
        'decode_config4_wide_rope': kv_bytes(g_lens.cpu(), 2, 128, 2),
        'decode_config1_simt_fp32': kv_bytes(c_lens.cpu(), 2, 64, 4),
        'rope_prefill_32x12x512x128': 2 * x.numel() * 2,
        'rms_norm_prefill_16384x1536': 2 * h.numel() * 2,
        'silu_mul_prefill_16384x8960': gate_up.numel() * 2 + gate_up.numel(),
        'contiguous_decode_qwen7b_geometry': kv_bytes(cc_lens, 4, 128, 2),
        'chunk_attention_qwen7b_geometry_t4': kv_bytes(ch_lens.cpu(), 4, 128, 2),
    }
    cc_lens = cc_lens.to(device)
    calls = {
        'decode_config4_wide_rope': lambda: cuda_attention.paged_decode_with_append(
            g_q, g_rows[:, 0], g_rows[:, 1], g_k, g_v, g_table, g_lens, max_context_len=int(g_table.shape[1] * 16),
            rope=(cos, sin)),
        'decode_config1_simt_fp32': lambda: cuda_attention.paged_decode_with_append(
            c_q, c_rows[:, 0], c_rows[:, 1], c_k, c_v, c_table, c_lens, max_context_len=int(c_table.shape[1] * 16)),
        'rope_prefill_32x12x512x128': lambda: apply_rope(x, cos, sin, start=0),
        'rms_norm_prefill_16384x1536': lambda: rms_norm(h, w, 1e-6),
        'silu_mul_prefill_16384x8960': lambda: silu_mul(gate_up),
        'contiguous_decode_qwen7b_geometry': lambda: cuda_attention.contiguous_decode_attention(
            cc_q, cc_k, cc_v, cc_lens),
        'chunk_attention_qwen7b_geometry_t4': lambda: cuda_attention.paged_chunk_attention(
            ch_q, ch_k, ch_v, ch_table, ch_lens),
        'chunk_attention_qwen7b_geometry_t4_rows': lambda: cuda_attention.paged_chunk_attention(
            ch_q, ch_k, ch_v, ch_table, ch_lens, kernel='rows'),
        'chunk_prefill_qwen15b_t256_after_1024': lambda: cuda_attention.paged_chunk_attention(
            cp_q, cp_k, cp_v, cp_table, cp_lens),
        'chunk_prefill_qwen15b_t256_after_1024_mma_sync': lambda: cuda_attention.paged_chunk_attention(
            cp_q, cp_k, cp_v, cp_table, cp_lens, kernel='mma_sync'),
        'chunk_prefill_qwen15b_t256_after_1024_rows': lambda: cuda_attention.paged_chunk_attention(
            cp_q, cp_k, cp_v, cp_table, cp_lens, kernel='rows'),
    }
    flops = {name: chunk_flops(cp_lens.cpu(), 256, 12, 128) for name in calls if name.startswith('chunk_prefill')}
    timings = {}
    stream = torch.cuda.Stream(device)
    calls = {name: fn for name, fn in calls.items() if args.kernels in name}
    for name, fn in calls.items():
        stream.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(stream):
            for _ in range(max(args.warmup, 1)):
                fn()
        torch.cuda.synchronize(device)
        # Back-to-back calls captured in one graph, so host overhead is not timed.
        calls_per_graph = max(1, min(args.steps, 20))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(calls_per_graph):
                fn()
        graph.replay()
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        start.record()
        for _ in range(reps):
            graph.replay()
        end.record()
        torch.cuda.synchronize(device)
        timings[name] = round(start.elapsed_time(end) * 1e3 / (reps * calls_per_graph), 2)
        del graph
    algorithmic['chunk_attention_qwen7b_geometry_t4_rows'] = algorithmic['chunk_attention_qwen7b_geometry_t4']
    gbs = {name: round(algorithmic[name] / (us * 1e3), 1) for name, us in timings.items() if name in algorithmic}
    tflops = {name: round(flops[name] / (us * 1e6), 1) for name, us in timings.items() if name in flops}
    return {'metric': 'per-call device time of this library\'s kernels on config-4 / config-1 shapes',
            'unit': 'us per call', 'values': timings,
            'algorithmic_gbs': gbs, 'algorithmic_tflops': tflops,
            'note': ('algorithmic bytes: K and V read once (decode, contiguous decode; the chunk entry counts '
                     'them once though each of its rows reads its own prefix), rows in and out (row kernels)'),
            'config': {'workload': 'kernels_qwen15b',
                       'timing': 'CUDA events around replays of a graph of back-to-back calls'}}


def main(argv=None):
    args = parse_args(argv)
    if args.workload == 'kernels_qwen15b':
        result = run_kernels(args)
    elif args.workload in GENERATE_WORKLOADS:
        if args.impl == 'reference':
            result = {'impl': 'reference', 'unavailable': 'the reference generates one request at a time on '
                      'the CPU path; a 1.5B-parameter batch-32 run is not a bounded sample'}
        else:
            result = run_generate(args)
    elif args.impl == 'reference':
        result = run_reference(args)
    else:
        result = run_ours(args)
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == '__main__':
    main()
