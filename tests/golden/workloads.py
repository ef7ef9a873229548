"""Benchmark workloads of the paged decode path: specs and on-device inputs.

Every workload is one decode step of one attention layer over a shared,
randomly permuted page pool: each sequence appends one new K/V token at
logical position ``L_i - 1`` and then attends over ``L_i`` cached tokens.
The named workloads follow the shapes, sizes and value distributions of the
configurations this path is measured on (seeded synthetic data; no dataset is
involved): Qwen2.5-0.5B head geometry in fp32/fp16/bf16, Qwen2.5-7B geometry at
batch 64 with 1k-4k tokens, Qwen3-8B geometry at 32k-131k tokens with 1% of K
rows scaled x8, Qwen2.5-72B geometry at batch 256 with lognormal lengths, and
odd shapes from the reference's CUDA tests. The ``*_small`` and ``edge_*``
entries keep a geometry at sizes the CPU oracle handles in milliseconds.

``make_workload`` builds a workload's inputs on a device with torch's seeded
generators -- the inputs ``bench.py`` times and the full-size GPU parity tests
check. ``tests/golden/cases.py`` builds the host-side (numpy) inputs of the
committed fixtures from the same specs. This module imports no oracle code.
"""
import math

# name -> spec. lens: ('uniform', lo, hi) | ('lognormal', median, sigma, lo, hi) | ('fixed', [..])
WORKLOADS = {
    # Qwen2.5-0.5B head geometry, fp32, 256-page pool.
    'qwen05b_fp32': dict(batch=4, q_heads=14, kv_heads=2, head_dim=64, block_size=16,
                         pool=('fixed_pages', 256), lens=('uniform', 1, 512),
                         dtype='float32', value_scale=1.0, seed=1001),
    'qwen05b_fp16': dict(batch=4, q_heads=14, kv_heads=2, head_dim=64, block_size=16,
                         pool=('fixed_pages', 256), lens=('uniform', 1, 512),
                         dtype='float16', value_scale=1.0, seed=1002),
    'qwen05b_bf16': dict(batch=4, q_heads=14, kv_heads=2, head_dim=64, block_size=16,
                         pool=('fixed_pages', 256), lens=('uniform', 1, 512),
                         dtype='bfloat16', value_scale=1.0, seed=1003),
    # Qwen2.5-7B geometry, bf16, pool 1.25x the pages in use.
    'qwen7b_bf16': dict(batch=64, q_heads=28, kv_heads=4, head_dim=128, block_size=16,
                        pool=('factor', 1.25), lens=('uniform', 1024, 4096),
                        dtype='bfloat16', value_scale=0.5, seed=2001),
    'qwen7b_bf16_small': dict(batch=3, q_heads=28, kv_heads=4, head_dim=128, block_size=16,
                              pool=('factor', 1.25), lens=('fixed', [1, 17, 300]),
                              dtype='bfloat16', value_scale=0.5, seed=2002),
    # Qwen3-8B long context, bf16, 1% of K rows scaled x8.
    'qwen3_8b_long_bf16': dict(batch=8, q_heads=32, kv_heads=8, head_dim=128, block_size=16,
                               pool=('factor', 1.0), lens=('uniform', 32768, 131072),
                               dtype='bfloat16', value_scale=1.0, k_outlier=(0.01, 8.0),
                               seed=3001),
    'qwen3_8b_bf16_small': dict(batch=2, q_heads=32, kv_heads=8, head_dim=128, block_size=16,
                                pool=('factor', 1.0), lens=('fixed', [700, 1029]),
                                dtype='bfloat16', value_scale=1.0, k_outlier=(0.01, 8.0),
                                seed=3002),
    # Qwen2.5-72B TP layer geometry, lognormal lengths.
    'qwen72b_bf16': dict(batch=256, q_heads=64, kv_heads=8, head_dim=128, block_size=16,
                         pool=('factor', 1.0), lens=('lognormal', 2048, 1.0, 16, 32768),
                         dtype='bfloat16', value_scale=1.0, seed=5001),
    'qwen72b_bf16_small': dict(batch=4, q_heads=64, kv_heads=8, head_dim=128, block_size=16,
                               pool=('factor', 1.0), lens=('fixed', [16, 33, 250, 64]),
                               dtype='bfloat16', value_scale=1.0, seed=5002),
    # Odd geometry from the reference's CUDA tests: page size 3/4, D 33/257, G 3/14.
    'edge_bs3_d33_fp32': dict(batch=3, q_heads=6, kv_heads=2, head_dim=33, block_size=3,
                              pool=('factor', 1.5), lens=('fixed', [2, 3, 65]),
                              dtype='float32', value_scale=1.0, seed=7001),
    'edge_bs4_d257_fp16': dict(batch=2, q_heads=14, kv_heads=1, head_dim=257, block_size=4,
                               pool=('factor', 1.5), lens=('fixed', [5, 33]),
                               dtype='float16', value_scale=1.0, seed=7002),
    'edge_bs64_d64_bf16': dict(batch=2, q_heads=4, kv_heads=4, head_dim=64, block_size=64,
                               pool=('factor', 2.0), lens=('fixed', [63, 129]),
                               dtype='bfloat16', value_scale=1.0, seed=7003),
}


def draw_lengths(spec, generator):
    """Context lengths [B] (int64, CPU) of a workload, drawn with a torch generator."""
    import torch
    batch = spec['batch']
    kind = spec['lens'][0]
    if kind == 'uniform':
        _, lo, hi = spec['lens']
        return torch.randint(lo, hi + 1, (batch,), generator=generator, dtype=torch.int64)
    if kind == 'lognormal':
        _, median, sigma, lo, hi = spec['lens']
        raw = torch.empty(batch, dtype=torch.float64).log_normal_(math.log(median), sigma,
                                                                   generator=generator)
        return raw.round().clamp(lo, hi).to(torch.int64)
    return torch.tensor(spec['lens'][1], dtype=torch.int64)


def make_workload(spec, q_heads, kv_heads, batch_slice, seed, device, value_seed=None):
    """Seeded synthetic inputs of the workload's shapes, built on ``device``.

    ``q_heads``/``kv_heads``/``batch_slice`` select a KV-head shard (the whole
    layer on one GPU: the spec's head counts and ``(0, batch)``). ``seed``
    draws the lengths and the page tables; ``value_seed`` (default ``seed +
    1``) draws q, K and V, so ranks can share one shape of work with their own
    values. Returns q
    [B, Hq, D], k_pool/v_pool [P, Hkv, bs, D] (before the append), k_new/v_new
    [B, Hkv, 1, D], block_table int32 [B, max_pages] (unused entries -1) and
    context_lens int32 [B] (after the append) on the device, plus host copies
    of the lengths and the table.
    """
    import torch
    dtype = {'bfloat16': torch.bfloat16, 'float16': torch.float16, 'float32': torch.float32}[spec['dtype']]
    cpu = torch.Generator().manual_seed(seed)
    lens = draw_lengths(spec, cpu)[batch_slice[0]:batch_slice[1]]
    bs, dim = spec['block_size'], spec['head_dim']
    pages = (lens + bs - 1) // bs
    total = int(pages.sum())
    kind, amount = spec['pool']
    num_pages = max(total, int(amount) if kind == 'fixed_pages' else int(math.ceil(total * amount)))
    perm = torch.randperm(num_pages, generator=cpu).to(torch.int32)
    table = torch.full((len(lens), int(pages.max())), -1, dtype=torch.int32)
    offset = 0
    for b, n in enumerate(pages.tolist()):
        table[b, :n] = perm[offset:offset + n]
        offset += n
    gen = torch.Generator(device=device).manual_seed(seed + 1 if value_seed is None else value_seed)
    scale = spec['value_scale']

    def normal(shape):
        out = torch.empty(shape, dtype=dtype, device=device)
        chunk = 1 << 26
        flat = out.view(-1)
        for start in range(0, flat.numel(), chunk):
            piece = torch.randn(min(chunk, flat.numel() - start), generator=gen, device=device)
            flat[start:start + piece.numel()] = piece.mul_(scale)
        return out

    pool_shape = (num_pages, kv_heads, bs, dim)
    k_pool = normal(pool_shape)
    v_pool = normal(pool_shape)
    if 'k_outlier' in spec:
        frac, factor = spec['k_outlier']
        mask = torch.rand((num_pages, kv_heads, bs), generator=gen, device=device) < frac
        k_pool[mask] *= factor
    return dict(
        q=normal((len(lens), q_heads, dim)),
        k_pool=k_pool, v_pool=v_pool,
        k_new=normal((len(lens), kv_heads, 1, dim)),
        v_new=normal((len(lens), kv_heads, 1, dim)),
        block_table=table.to(device), context_lens=lens.to(torch.int32).to(device),
        host_lens=lens.clone(), host_table=table.clone(), dtype=dtype)
