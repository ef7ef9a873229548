"""Host-side (numpy) inputs of the paged-decode workloads, for the fixtures and tests.

The workload specs live in ``tests/golden/workloads.py`` (re-exported here as
``WORKLOADS``). ``make_inputs`` draws a workload's inputs with numpy's PCG64
``default_rng``, for the committed golden fixtures and the CPU-sized parity
tests; the fixtures store a SHA-256 of the generated arrays so that a change
in the generator is caught instead of silently comparing different data.
"""
import hashlib
import math

import numpy as np

from oracle.dtypes import from_float32
from tests.golden.workloads import WORKLOADS  # re-exported


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
