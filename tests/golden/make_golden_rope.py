"""Generate the RoPE golden fixture by running micro-vllm's own reference code.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden_rope.py REFERENCE_ROOT

For each (dtype, head_dim) case this calls the reference's ``rope_cos_sin``
(src/micro_vllm/model.py:79-98) on a set of positions with theta 1e6 (Qwen2)
and its ``apply_rope`` (model.py:110-123) on seeded q and K rows at those
positions, and stores the inputs, the tables and the outputs as storage
arrays in ``rope_cases.npz``. Nothing at test time reads the reference.
"""
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden.cases import _normal  # noqa: E402

ROPE_CASES = (('float32', 64), ('float16', 64), ('bfloat16', 128), ('float16', 128), ('bfloat16', 256))
POSITIONS = np.array([0, 1, 2, 15, 16, 1023, 4095, 32767, 131071], dtype=np.int64)
THETA = 1000000.0


def _torch(array, dtype):
    import torch
    if dtype == 'bfloat16':
        return torch.from_numpy(array.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(array.copy())


def _numpy(tensor, dtype):
    import torch
    if dtype == 'bfloat16':
        return tensor.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return tensor.contiguous().numpy().copy()


def run_reference():
    import torch
    from micro_vllm import model

    fixture = {'positions': POSITIONS, 'theta': np.array(THETA)}
    for index, (dtype, dim) in enumerate(ROPE_CASES):
        tdtype = {'float32': torch.float32, 'float16': torch.float16, 'bfloat16': torch.bfloat16}[dtype]
        rng = np.random.default_rng(1234 + index)
        n = len(POSITIONS)
        q = _normal(rng, (n, 4, dim), 1.0, dtype)      # [positions, heads, D]
        k = _normal(rng, (n, 2, dim), 1.0, dtype)
        cos, sin = model.rope_cos_sin(torch.from_numpy(POSITIONS)[None], dim, THETA, dtype=tdtype)
        query = _torch(q, dtype).transpose(0, 1)[None]   # [1, heads, tokens, D]
        key = _torch(k, dtype).transpose(0, 1)[None]
        rq, rk = model.apply_rope(query, key, cos, sin)
        tag = f'{dtype}_{dim}'
        fixture[f'{tag}_q'] = q
        fixture[f'{tag}_k'] = k
        fixture[f'{tag}_cos'] = _numpy(cos[0], dtype)
        fixture[f'{tag}_sin'] = _numpy(sin[0], dtype)
        fixture[f'{tag}_q_out'] = _numpy(rq[0].transpose(0, 1), dtype)
        fixture[f'{tag}_k_out'] = _numpy(rk[0].transpose(0, 1), dtype)
    return fixture


def main(reference_root):
    sys.dont_write_bytecode = True
    os.environ.setdefault('PYTHONDONTWRITEBYTECODE', '1')
    sys.path.insert(0, str(Path(reference_root) / 'src'))
    fixture = run_reference()
    np.savez_compressed(HERE / 'rope_cases.npz', **fixture)
    print(f'rope_cases.npz: {len(ROPE_CASES)} cases x {len(POSITIONS)} positions')


if __name__ == '__main__':
    source = sys.argv[1] if len(sys.argv) > 1 else os.environ.get('MICRO_VLLM_REFERENCE_ROOT')
    if not source:
        raise SystemExit('usage: python tests/golden/make_golden_rope.py REFERENCE_ROOT')
    main(source)
