"""Pin the RoPE oracle and the host table builder against micro-vllm's own code.

tests/golden/rope_cases.npz was produced by tests/golden/make_golden_rope.py,
which runs the reference's rope_cos_sin and apply_rope
(src/micro_vllm/model.py:79-123). The known-answer cases restate the
reference's own RoPE tests (test/test_rope.py:20-64).
"""
from pathlib import Path

import numpy as np
import pytest

from oracle import apply_rope
from oracle.dtypes import from_float32, to_float32
from tests.golden.make_golden_rope import POSITIONS, ROPE_CASES, THETA

FIXTURE = Path(__file__).resolve().parent / 'golden' / 'rope_cases.npz'


def load():
    with np.load(FIXTURE) as data:
        return {key: data[key] for key in data.files}


@pytest.mark.parametrize('dtype,dim', ROPE_CASES)
def test_oracle_matches_the_reference_bit_for_bit(dtype, dim):
    f = load()
    tag = f'{dtype}_{dim}'
    cos, sin = f[f'{tag}_cos'][:, None, :], f[f'{tag}_sin'][:, None, :]
    for name in ('q', 'k'):
        out = apply_rope(f[f'{tag}_{name}'], cos, sin, dtype)
        assert np.array_equal(out.view(np.uint8), f[f'{tag}_{name}_out'].view(np.uint8)), name


@pytest.mark.parametrize('dtype,dim', ROPE_CASES)
def test_host_tables_equal_the_reference_tables(dtype, dim):
    import torch

    from micro_vllm_b200.rope import rope_tables
    f = load()
    tdtype = {'float32': torch.float32, 'float16': torch.float16, 'bfloat16': torch.bfloat16}[dtype]
    cos, sin = rope_tables(int(POSITIONS.max()) + 1, dim, float(f['theta']), dtype=tdtype, device='cpu')
    pick = torch.from_numpy(POSITIONS)
    for table, name in ((cos, 'cos'), (sin, 'sin')):
        rows = table[pick]
        bits = rows.view(torch.int16).numpy().view(np.uint16) if dtype == 'bfloat16' else rows.numpy()
        assert np.array_equal(bits.view(np.uint8), f[f'{dtype}_{dim}_{name}'].view(np.uint8))
    assert float(f['theta']) == THETA


def test_known_answers_from_the_reference_tests():
    # rotate_half maps [1, 2, 3, 4] to [-3, -4, 1, 2] (test_rope.py:20-24).
    from oracle.rope import rotate_half
    assert rotate_half(np.array([1., 2., 3., 4.], dtype=np.float32)).tolist() == [-3., -4., 1., 2.]
    # A quarter turn (cos 0, sin 1) is rotate_half itself (test_rope.py:35-46).
    q = np.arange(1., 17., dtype=np.float32).reshape(4, 4)
    out = apply_rope(q, np.zeros((1, 4), np.float32), np.ones((1, 4), np.float32), 'float32')
    assert out.tolist() == [[-3., -4., 1., 2.], [-7., -8., 5., 6.], [-11., -12., 9., 10.],
                            [-15., -16., 13., 14.]]
    # Position 0 is the identity in every dtype (test_rope.py:48-64).
    for dtype in ('float32', 'float16', 'bfloat16'):
        x = from_float32(np.random.default_rng(13).standard_normal((3, 8), dtype=np.float32), dtype)
        one = from_float32(np.ones((1, 8), np.float32), dtype)
        zero = from_float32(np.zeros((1, 8), np.float32), dtype)
        assert np.array_equal(to_float32(apply_rope(x, one, zero, dtype), dtype), to_float32(x, dtype))


def test_rope_tables_reject_what_the_reference_rejects():
    from micro_vllm_b200.rope import rope_tables
    import torch
    for dim, theta in ((0, 1e4), (3, 1e4), (4, 0.), (4, -1.), (4, float('nan')), (4, float('inf'))):
        with pytest.raises(ValueError):
            rope_tables(4, dim, theta, dtype=torch.float32, device='cpu')
