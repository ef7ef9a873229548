"""Batched greedy generation on the GPU against the reference's own greedy loop.

tests/golden/tiny_qwen2_*.npz hold the tokens micro-vllm's ``_greedy_decode``
(paged cache, page size 16, fp32, CPU) produced for each prompt on its own,
and its prefill logits (tests/golden/make_golden_generate.py). Here all
prompts of a case run as one batch through ``generate.greedy_decode``: batched
prefill, then CUDA-graph decode steps whose attention is the one-call
RoPE + append + paged decode kernel.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.golden.model_cases import MODEL_CASES, make_prompts, make_weights, model_config

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / 'golden'


def _load(name):
    with np.load(GOLDEN / f'{name}.npz') as f:
        return {k: f[k] for k in f.files}


def _weights(name, dtype=torch.float32):
    return {k: torch.from_numpy(v).to(dtype).cuda() for k, v in make_weights(name).items()}


@pytest.mark.parametrize('name', list(MODEL_CASES))
@pytest.mark.parametrize('use_graph', [True, False])
def test_batched_greedy_tokens_match_the_reference_per_prompt(name, use_graph):
    from micro_vllm_b200.generate import greedy_decode
    fixture = _load(name)
    prompts = torch.from_numpy(make_prompts(name)).cuda()
    tokens = greedy_decode(_weights(name), model_config(name), prompts, MODEL_CASES[name]['new_tokens'],
                           use_graph=use_graph)
    assert tokens.shape == fixture['tokens'].shape and tokens.dtype == torch.long
    assert np.array_equal(tokens.cpu().numpy(), fixture['tokens'])


@pytest.mark.parametrize('name', list(MODEL_CASES))
def test_prefill_logits_match_the_reference(name):
    from micro_vllm_b200.runtime import prepare_model
    fixture = _load(name)
    model = prepare_model(_weights(name), model_config(name))
    prompts = torch.from_numpy(make_prompts(name)).cuda()
    cache = model.allocate_cache(prompts.shape[0], prompts.shape[1] + 4, shuffle_seed=3)
    logits = model.prefill(prompts, cache).cpu().numpy()
    np.testing.assert_allclose(logits, fixture['prefill_logits'], rtol=1e-4, atol=1e-4)
    assert cache.sequence_length == prompts.shape[1]
    assert cache.lengths.tolist() == [prompts.shape[1]] * prompts.shape[0]


def test_eos_cuts_each_sequence_after_its_first_eos():
    from micro_vllm_b200.generate import greedy_decode
    name = 'tiny_qwen2_fp32'
    fixture = _load(name)['tokens']
    eos = int(fixture[0, 5])
    prompts = torch.from_numpy(make_prompts(name)).cuda()
    rows = greedy_decode(_weights(name), model_config(name), prompts, fixture.shape[1], eos_token_id=eos)
    for row, expected in zip(rows, fixture):
        hits = np.nonzero(expected == eos)[0]
        cut = expected[:hits[0] + 1] if len(hits) else expected
        assert row.cpu().numpy().tolist() == cut.tolist()


def test_bf16_generation_runs_on_the_tensor_core_decode_path():
    from micro_vllm_b200.generate import GreedyDecoder
    from micro_vllm_b200.runtime import prepare_model
    name = 'tiny_qwen2_tied'
    model = prepare_model(_weights(name, torch.bfloat16), model_config(name))
    prompts = torch.from_numpy(make_prompts(name)).cuda()
    decoder = GreedyDecoder(model, prompts.shape[0], prompts.shape[1] + 8)
    assert model._steps[0].plan[0] == 'tma_mma' and model._steps[0]._rope_in_kernel
    tokens = decoder.run(prompts, 8)
    assert tokens.shape == (prompts.shape[0], 8)
    assert int(tokens.min()) >= 0 and int(tokens.max()) < model.vocab
    # The graph-replayed steps equal eager steps on the same state.
    eager = GreedyDecoder(model, prompts.shape[0], prompts.shape[1] + 8, use_graph=False)
    assert torch.equal(eager.run(prompts, 8), tokens)
