"""Generate the golden fixtures by running micro-vllm's own Python reference.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden.py REFERENCE_ROOT

For each workload in ``GOLDEN_CASES`` this builds, per sequence, a reference
``PagedKVCache`` over ONE shared page pool (its dataclass constructor accepts
externally owned pools: src/micro_vllm/paged_kv_cache.py:43-51), appends the
new K/V token with the reference's CPU append (``_append_cpu``,
paged_kv_cache.py:151-161), gathers the sequence (paged_kv_cache.py:188-193)
and calls ``causal_attention`` (attention.py:57-94) with
``past_length = L - 1``. It stores the reference output and SHA-256 digests of
the pools after the append. Inputs are not stored; ``cases.make_inputs``
regenerates them and the fixture records their digest.

Nothing at test time reads the reference checkout: the fixtures are committed.
"""
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden.cases import WORKLOADS, array_digest, input_digest, make_inputs  # noqa: E402

GOLDEN_CASES = (
    'qwen05b_fp32', 'qwen05b_fp16', 'qwen05b_bf16',
    'qwen7b_bf16_small', 'qwen3_8b_bf16_small', 'qwen72b_bf16_small',
    'edge_bs3_d33_fp32', 'edge_bs4_d257_fp16', 'edge_bs64_d64_bf16',
)


def _torch_tensor(array, dtype_name):
    import torch
    if dtype_name == 'bfloat16':
        return torch.from_numpy(array.view(np.int16).copy()).view(torch.bfloat16)
    return torch.from_numpy(array.copy())


def _to_numpy(tensor, dtype_name):
    import torch
    if dtype_name == 'bfloat16':
        return tensor.contiguous().view(torch.int16).numpy().view(np.uint16).copy()
    return tensor.contiguous().numpy().copy()


def run_reference(name):
    import torch
    from micro_vllm.attention import causal_attention
    from micro_vllm.paged_kv_cache import PagedKVCache

    inputs = make_inputs(name)
    spec = inputs['spec']
    dtype = spec['dtype']
    bs = spec['block_size']
    key_pool = _torch_tensor(inputs['key_pool'], dtype)
    value_pool = _torch_tensor(inputs['value_pool'], dtype)
    q = _torch_tensor(inputs['q'], dtype)
    key_new = _torch_tensor(inputs['key_new'], dtype)
    value_new = _torch_tensor(inputs['value_new'], dtype)
    outputs = []
    for b in range(spec['batch']):
        length = int(inputs['context_lens'][b])
        used = -(-length // bs)
        ids = tuple(int(x) for x in inputs['block_table'][b, :used])
        cache = PagedKVCache((key_pool,), (value_pool,), [length - 1], ids,
                             torch.tensor(ids, dtype=torch.int64))
        cache.append(0, key_new[b:b + 1], value_new[b:b + 1])
        k, v = cache.gather(0)
        out = causal_attention(q[b:b + 1, :, None, :], k, v, past_length=length - 1)
        outputs.append(out[0, :, 0, :])
    out = torch.stack(outputs)
    return dict(
        input_digest=np.array(input_digest(inputs)),
        out=_to_numpy(out, dtype),
        key_pool_digest=np.array(array_digest(_to_numpy(key_pool, dtype))),
        value_pool_digest=np.array(array_digest(_to_numpy(value_pool, dtype))),
        dtype=np.array(dtype),
    )


def main(reference_root):
    sys.dont_write_bytecode = True
    os.environ.setdefault('PYTHONDONTWRITEBYTECODE', '1')
    sys.path.insert(0, str(Path(reference_root) / 'src'))
    for name in GOLDEN_CASES:
        assert name in WORKLOADS, name
        fixture = run_reference(name)
        path = HERE / f'{name}.npz'
        np.savez_compressed(path, **fixture)
        print(f'{name}: out {fixture["out"].shape} {fixture["out"].dtype} -> {path.name}')


if __name__ == '__main__':
    source = sys.argv[1] if len(sys.argv) > 1 else os.environ.get('MICRO_VLLM_REFERENCE_ROOT')
    if not source:
        raise SystemExit('usage: python tests/golden/make_golden.py REFERENCE_ROOT')
    main(source)
