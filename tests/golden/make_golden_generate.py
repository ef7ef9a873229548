"""Generate the batched-generation golden fixtures with micro-vllm's own code.

Run in a container where the reference checkout is present:

    python tests/golden/make_golden_generate.py REFERENCE_ROOT

For each model case, every prompt is decoded on its own (the reference is
batch 1) by the reference's greedy loop over a paged KV cache
(``generate._greedy_decode`` with ``kv_cache='paged'``, page size 16, the
torch attention backend on CPU, fp32; src/micro_vllm/generate.py:82-107),
and its prefill logits of the last prompt position come from the reference's
``forward`` (model.py:310-320). The fixture stores the generated token IDs
and those logits; weights and prompts are rebuilt from seeds at test time
(``model_cases``) and their digests are stored to catch a generator change.
"""
import hashlib
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden.model_cases import MODEL_CASES, make_prompts, make_weights, model_config  # noqa: E402


def weights_digest(weights):
    h = hashlib.sha256()
    for name in sorted(weights):
        h.update(name.encode())
        h.update(np.ascontiguousarray(weights[name]).tobytes())
    return h.hexdigest()


def run_reference(name):
    import torch
    from micro_vllm import generate
    from micro_vllm.model import forward, prepare_model

    case = MODEL_CASES[name]
    config = model_config(name)
    weights_np = make_weights(name)
    weights = {k: torch.from_numpy(v.copy()) for k, v in weights_np.items()}
    prompts = make_prompts(name)
    tokens, logits = [], []
    prepared = prepare_model(weights, config, attention_backend='torch')
    for row in prompts:
        ids = torch.from_numpy(row.copy())[None]
        out = generate._greedy_decode(ids, weights, config, case['new_tokens'], eos_token_id=None,
                                      attention_backend='torch', kv_cache='paged', page_size=16)
        assert out.shape == (case['new_tokens'],)
        tokens.append(out.numpy())
        logits.append(forward(ids, prepared, logits_to_keep=1)[0, -1].numpy())
    return dict(tokens=np.stack(tokens), prefill_logits=np.stack(logits),
                weights_digest=np.array(weights_digest(weights_np)),
                prompts_digest=np.array(hashlib.sha256(prompts.tobytes()).hexdigest()))


def main(reference_root):
    sys.dont_write_bytecode = True
    os.environ.setdefault('PYTHONDONTWRITEBYTECODE', '1')
    sys.path.insert(0, str(Path(reference_root) / 'src'))
    for name in MODEL_CASES:
        fixture = run_reference(name)
        np.savez_compressed(HERE / f'{name}.npz', **fixture)
        print(f'{name}: tokens {fixture["tokens"].shape}')


if __name__ == '__main__':
    source = sys.argv[1] if len(sys.argv) > 1 else os.environ.get('MICRO_VLLM_REFERENCE_ROOT')
    if not source:
        raise SystemExit('usage: python tests/golden/make_golden_generate.py REFERENCE_ROOT')
    main(source)
