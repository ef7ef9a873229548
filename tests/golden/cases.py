"""Seeded paged-decode workloads shared by the golden fixtures, tests and bench.

Every workload is one decode step of one attention layer over a shared,
randomly permuted page pool: each sequence appends one new K/V token at
logical position ``L_i - 1`` and then attends over ``L_i`` cached tokens.

The named workloads follow the shapes, sizes and value distributions of the
benchmark configurations this path is measured on (seeded synthetic data; no
dataset is involved). The small ``edge_*`` and ``*_small`` cases keep the
same head geometry at sizes the CPU oracle and the committed fixtures handle
in milliseconds.

Inputs are generated with numpy's PCG64 ``default_rng``; the fixtures store a
SHA-256 of the generated arrays so that a change in the generator is caught
instead of silently comparing different data.
"""
import hashlib
import math

import numpy as np

from oracle.dtypes import from_float32

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


def _draw_lengths(rng, spec):
    kind = spec['lens'][0]
    batch = spec['batch']
    if kind == 'fixed':
        lens = np.asarray(spec['lens'][1], dtype=np.int64)
        assert lens.shape == (batch,)
        return lens
    if kind == 'uniform':
        _, lo, hi = spec['lens']
        return rng.integers(lo, hi + 1, size=batch, dtype=np.int64)
    if kind == 'lognormal':
        _, median, sigma, lo, hi = spec['lens']
        raw = rng.lognormal(mean=math.log(median), sigma=sigma, size=batch)
        return np.clip(np.round(raw), lo, hi).astype(np.int64)
    raise ValueError(kind)


def _normal(rng, shape, scale, dtype):
    values = rng.standard_normal(size=shape, dtype=np.float32)
    if scale != 1.0:
        values *= np.float32(scale)
    return from_float32(values, dtype)


def make_inputs(name_or_spec):
    """Generate one workload's inputs as numpy arrays (storage dtypes).

    Returns dict with q [B,Hq,D], key_pool/value_pool [P,Hkv,bs,D] (contents
    before the append), key_new/value_new [B,Hkv,1,D], block_table int32
    [B, max_pages] (unused entries -1), context_lens int32 [B] (after the
    append), and the spec.
    """
    spec = WORKLOADS[name_or_spec] if isinstance(name_or_spec, str) else name_or_spec
    rng = np.random.default_rng(spec['seed'])
    batch, hq, hkv, dim, bs = (spec[k] for k in
                               ('batch', 'q_heads', 'kv_heads', 'head_dim', 'block_size'))
    dtype = spec['dtype']
    lens = _draw_lengths(rng, spec)
    pages = -(-lens // bs)
    total = int(pages.sum())
    kind, amount = spec['pool']
    num_pages = int(amount) if kind == 'fixed_pages' else int(math.ceil(total * amount))
    num_pages = max(num_pages, total)
    perm = rng.permutation(num_pages).astype(np.int64)
    max_pages = int(pages.max())
    table = np.full((batch, max_pages), -1, dtype=np.int32)
    offset = 0
    for b in range(batch):
        table[b, :pages[b]] = perm[offset:offset + pages[b]]
        offset += pages[b]
    scale = spec['value_scale']
    pool_shape = (num_pages, hkv, bs, dim)
    key_pool = _normal(rng, pool_shape, scale, dtype)
    value_pool = _normal(rng, pool_shape, scale, dtype)
    if 'k_outlier' in spec:
        frac, factor = spec['k_outlier']
        mask = rng.random(size=(num_pages, bs, hkv)) < frac   # rows = (page, slot, head)
        from oracle.dtypes import to_float32
        widened = to_float32(key_pool, dtype)
        widened[mask.transpose(0, 2, 1)] *= np.float32(factor)
        key_pool = from_float32(widened, dtype)
    q = _normal(rng, (batch, hq, dim), scale, dtype)
    key_new = _normal(rng, (batch, hkv, 1, dim), scale, dtype)
    value_new = _normal(rng, (batch, hkv, 1, dim), scale, dtype)
    return dict(spec=spec, q=q, key_pool=key_pool, value_pool=value_pool,
                key_new=key_new, value_new=value_new, block_table=table,
                context_lens=lens.astype(np.int32))


def input_digest(inputs) -> str:
    """SHA-256 over every generated array, in a fixed order."""
    digest = hashlib.sha256()
    for key in ('q', 'key_pool', 'value_pool', 'key_new', 'value_new',
                'block_table', 'context_lens'):
        array = np.ascontiguousarray(inputs[key])
        digest.update(key.encode())
        digest.update(str(array.dtype).encode())
        digest.update(str(array.shape).encode())
        digest.update(array.tobytes())
    return digest.hexdigest()


def array_digest(array) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


def algorithmic_bytes(spec, context_lens, include_append=True):
    """Bytes one decode step must move, by the roofline definition of this path.

    sum_i 2*Hkv*L_i*D*s_kv (K and V read once) + B*Hq*D*(s_q + s_o) +
    sum_i ceil(L_i/bs)*s_idx + 4*B (context lengths), plus 4*B*Hkv*D*s_kv for
    the append (read new K and V, write them into pages).
    """
    elem = 4 if spec['dtype'] == 'float32' else 2
    lens = np.asarray(context_lens, dtype=np.int64)
    b, hq, hkv, d, bs = (spec[k] for k in ('batch', 'q_heads', 'kv_heads', 'head_dim',
                                           'block_size'))
    kv = int((2 * hkv * lens * d * elem).sum())
    qo = b * hq * d * 2 * elem
    idx = int((-(-lens // bs)).sum()) * 4
    total = kv + qo + idx + 4 * b
    if include_append:
        total += 4 * b * hkv * d * elem
    return total
