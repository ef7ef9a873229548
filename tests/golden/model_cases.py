"""Seeded random-init Qwen2 models for the batched generation tests.

A model case is a Qwen2 configuration (as plain attributes, the ones
micro-vllm's forward reads: src/micro_vllm/runtime.py:140-165,
model.py:248-266), a weight seed and a set of equal-length prompts. Weights are
drawn with numpy's PCG64 ``default_rng`` from N(0, std^2) in fp32 (RMSNorm
scales from 1 + N(0, std^2)), so the fixtures need not store them: the tests
and the golden generator rebuild the same arrays.
"""
from types import SimpleNamespace

import numpy as np

MODEL_CASES = {
    # Two layers, 4 query / 2 KV heads of 64, pages crossed during prefill and decode.
    'tiny_qwen2_fp32': dict(
        config=dict(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
                    num_key_value_heads=2, vocab_size=1000, max_position_embeddings=512,
                    rope_theta=1000000.0, rms_norm_eps=1e-6, tie_word_embeddings=False),
        weight_seed=7, weight_std=0.08, prompt_seed=11, batch=3, prompt_len=37, new_tokens=20,
        dtype='float32'),
    # Tied embeddings, GQA group 3, head_dim 128 (the tensor-core decode shapes in bf16).
    'tiny_qwen2_tied': dict(
        config=dict(num_hidden_layers=3, hidden_size=384, intermediate_size=768, num_attention_heads=3,
                    num_key_value_heads=1, vocab_size=777, max_position_embeddings=256,
                    rope_theta=10000.0, rms_norm_eps=1e-6, tie_word_embeddings=True),
        weight_seed=8, weight_std=0.06, prompt_seed=12, batch=2, prompt_len=16, new_tokens=17,
        dtype='float32'),
}


# The accelerated tiny Qwen2 of micro-vllm's paged-forward GPU test
# (test/test_accelerated_generation.py:17-28): 2 layers, 14 query / 2 KV heads of
# 64, intermediate 128, vocabulary 128, tied embeddings. Weights here are seeded
# numpy draws rather than the Hugging Face initialisation.
CALL_SITE_CONFIG = dict(num_hidden_layers=2, hidden_size=896, intermediate_size=128, num_attention_heads=14,
                        num_key_value_heads=2, vocab_size=128, max_position_embeddings=128,
                        rope_theta=10000.0, rms_norm_eps=1e-6, tie_word_embeddings=True)

def model_config(name):
    """The case's configuration as an attribute object (no transformers needed)."""
    return config_object(MODEL_CASES[name]['config'])


def config_object(config):
    """A Qwen2 configuration dict as the attribute object micro-vllm's forward reads."""
    c = dict(config)
    return SimpleNamespace(model_type='qwen2', hidden_act='silu', rope_scaling=None, use_sliding_window=False,
                           layer_types=['full_attention'] * c['num_hidden_layers'], head_dim=None,
                           partial_rotary_factor=1.0, **c)


def make_weights(name):
    """name -> fp32 numpy array, in the checkpoint naming micro-vllm reads."""
    case = MODEL_CASES[name]
    return weights_for(case['config'], case['weight_seed'], case['weight_std'])


def weights_for(c, seed, std):
    """Seeded N(0, std^2) weights (RMSNorm scales 1 + N(0, std^2)) of a Qwen2 config dict."""
    rng = np.random.default_rng(seed)
    std = np.float32(std)
    hidden, inter = c['hidden_size'], c['intermediate_size']
    dim = hidden // c['num_attention_heads']
    kv = c['num_key_value_heads'] * dim

    def normal(*shape):
        return rng.standard_normal(size=shape, dtype=np.float32) * std

    weights = {'model.embed_tokens.weight': normal(c['vocab_size'], hidden)}
    for i in range(c['num_hidden_layers']):
        p = f'model.layers.{i}.'
        weights.update({
            p + 'input_layernorm.weight': 1 + normal(hidden),
            p + 'post_attention_layernorm.weight': 1 + normal(hidden),
            p + 'self_attn.q_proj.weight': normal(hidden, hidden),
            p + 'self_attn.k_proj.weight': normal(kv, hidden),
            p + 'self_attn.v_proj.weight': normal(kv, hidden),
            p + 'self_attn.q_proj.bias': normal(hidden),
            p + 'self_attn.k_proj.bias': normal(kv),
            p + 'self_attn.v_proj.bias': normal(kv),
            p + 'self_attn.o_proj.weight': normal(hidden, hidden),
            p + 'mlp.gate_proj.weight': normal(inter, hidden),
            p + 'mlp.up_proj.weight': normal(inter, hidden),
            p + 'mlp.down_proj.weight': normal(hidden, inter),
        })
    weights['model.norm.weight'] = 1 + normal(hidden)
    if not c['tie_word_embeddings']:
        weights['lm_head.weight'] = normal(c['vocab_size'], hidden)
    return weights


def make_prompts(name):
    case = MODEL_CASES[name]
    rng = np.random.default_rng(case['prompt_seed'])
    return rng.integers(0, case['config']['vocab_size'], size=(case['batch'], case['prompt_len']),
                        dtype=np.int64)
