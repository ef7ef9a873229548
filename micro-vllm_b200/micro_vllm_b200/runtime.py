"""Batched Qwen2 inference over a paged KV cache, built around the decode step.

The reference's runtime binds a checkpoint once (``prepare_model``,
src/micro_vllm/runtime.py:140-165) and runs one request at a time
(runtime.py:82-85). This module keeps its layer math -- RMSNorm with fp32
statistics, Q/K/V projections with bias, rotate-half RoPE, grouped attention,
bias-free output projection, SiLU-gated MLP (src/micro_vllm/model.py:25-165,
189-241) -- for a batch of B requests of equal prompt length:

* ``prefill``: the prompt of every sequence in one pass; RoPE and the cache
  append run as this library's kernels; the first chunk's self-attention is
  the library SDPA kernel, a chunk after cached tokens attends its causal
  prefix straight from the pages (``paged_chunk_attention``).
* ``decode``: one token per sequence; each layer's attention is one
  ``PagedDecodeStep`` call that rotates q and the new K (RoPE), appends K/V
  and attends over the pages in one kernel (plus the split merge).

Projections are library GEMMs (cuBLAS), Q/K/V and gate/up weights
concatenated once so each is one GEMM, with the residual adds in the GEMM
epilogue (addmm); RMSNorm and SiLU-gating are this library's fused row
kernels (``row_ops``). ``decode`` has static shapes and allocates nothing but its outputs, so
the greedy loop captures it in a CUDA graph.
"""
from collections.abc import Mapping

import torch
import torch.nn.functional as F

from .cuda_attention import PagedDecodeStep, paged_chunk_attention
from .paged_kv_cache import BatchedPagedKVCache
from .rope import apply_rope, rope_tables
from .row_ops import rms_norm, silu_mul


def _theta(config):
    theta = getattr(config, 'rope_theta', None)
    if theta is None:
        theta = (getattr(config, 'rope_parameters', None) or {}).get('rope_theta')
    if theta is None:
        raise ValueError('config must give rope_theta')
    return float(theta)


def _check_config(config):
    """The architecture subset the reference's forward accepts (model.py:247-266)."""
    scaling = getattr(config, 'rope_scaling', None)
    if scaling is not None and scaling.get('rope_type', 'default') != 'default':
        raise ValueError('forward supports Qwen2 with SiLU and unscaled RoPE')
    if config.model_type != 'qwen2' or config.hidden_act != 'silu':
        raise ValueError('forward supports Qwen2 with SiLU and unscaled RoPE')
    if getattr(config, 'use_sliding_window', False) or any(
            kind != 'full_attention' for kind in getattr(config, 'layer_types', ())):
        raise ValueError('forward currently supports full attention layers only')
    if (config.hidden_size % config.num_attention_heads
            or config.num_attention_heads % config.num_key_value_heads):
        raise ValueError('layer count, hidden width, and head counts must be positive and compatible')
    head_dim = config.hidden_size // config.num_attention_heads
    if (getattr(config, 'head_dim', None) not in (None, head_dim)
            or getattr(config, 'partial_rotary_factor', 1.0) != 1.0 or head_dim % 2):
        raise ValueError('forward requires full-head RoPE with the standard head dimension')
    return head_dim


class PreparedModel:
    """A Qwen2 checkpoint bound for batched prefill and decode over a paged cache."""

    def __init__(self, weights: Mapping[str, torch.Tensor], config):
        self.head_dim = _check_config(config)
        self.num_heads = config.num_attention_heads
        self.num_kv_heads = config.num_key_value_heads
        self.hidden = config.hidden_size
        self.eps = float(config.rms_norm_eps)
        self.vocab = config.vocab_size
        self.num_layers = config.num_hidden_layers
        self.max_positions = config.max_position_embeddings
        embedding = weights['model.embed_tokens.weight']
        self.embedding = embedding
        self.dtype, self.device = embedding.dtype, embedding.device
        if self.device.type != 'cuda':
            raise ValueError('the batched runtime requires CUDA weights')
        self.final_norm = weights['model.norm.weight']
        self.output = embedding if config.tie_word_embeddings else weights['lm_head.weight']
        self.layers = []
        for i in range(self.num_layers):
            p = f'model.layers.{i}.'
            w = {name: weights[p + name] for name in (
                'input_layernorm.weight', 'post_attention_layernorm.weight', 'self_attn.o_proj.weight',
                'mlp.down_proj.weight')}
            w['qkv'] = torch.cat([weights[p + f'self_attn.{x}_proj.weight'] for x in 'qkv'], dim=0).contiguous()
            w['qkv_bias'] = torch.cat([weights[p + f'self_attn.{x}_proj.bias'] for x in 'qkv']).contiguous()
            w['gate_up'] = torch.cat([weights[p + 'mlp.gate_proj.weight'],
                                      weights[p + 'mlp.up_proj.weight']], dim=0).contiguous()
            self.layers.append(w)
        self.cos, self.sin = rope_tables(self.max_positions, self.head_dim, _theta(config), dtype=self.dtype,
                                         device=self.device)
        self._steps = None

    def allocate_cache(self, batch_size, capacity, *, page_size=16, shuffle_seed=None):
        return BatchedPagedKVCache.allocate(
            num_layers=self.num_layers, batch_size=batch_size, capacity=capacity,
            num_kv_heads=self.num_kv_heads, head_dim=self.head_dim, dtype=self.dtype, device=self.device,
            page_size=page_size, shuffle_seed=shuffle_seed)

    def bind(self, cache: BatchedPagedKVCache):
        """One PagedDecodeStep per layer over this cache (RoPE fused), reused every step."""
        self._steps = [PagedDecodeStep(*cache.pools(i), cache.block_table, num_q_heads=self.num_heads,
                                       max_context_len=cache.capacity, rope=(self.cos, self.sin))
                       for i in range(self.num_layers)]
        self._cache = cache
        return self._steps

    def _mlp(self, x, w):
        # Residual adds ride in the GEMM epilogue (addmm: x + h W^T).
        h = rms_norm(x, w['post_attention_layernorm.weight'], self.eps)
        act = silu_mul(F.linear(h, w['gate_up']))
        flat = act.reshape(-1, act.shape[-1])
        return torch.addmm(x.reshape(-1, x.shape[-1]), flat, w['mlp.down_proj.weight'].t()).view(x.shape)

    def _logits(self, x):
        return F.linear(rms_norm(x, self.final_norm, self.eps), self.output)

    @torch.inference_mode()
    def prefill(self, input_ids: torch.Tensor, cache: BatchedPagedKVCache) -> torch.Tensor:
        """Run [B, T] prompt tokens from the cache's current length; logits of the last position."""
        batch, tokens = input_ids.shape
        start = cache.sequence_length
        if start + tokens > min(cache.capacity, self.max_positions):
            raise ValueError('sequence length exceeds the cache capacity or the configured context length')
        hq, hkv, d = self.num_heads, self.num_kv_heads, self.head_dim
        ends = cache.lengths + tokens  # each sequence's length after the chunk
        x = F.embedding(input_ids, self.embedding)
        for i, w in enumerate(self.layers):
            h = rms_norm(x, w['input_layernorm.weight'], self.eps)
            qkv = F.linear(h, w['qkv'], w['qkv_bias']).view(batch, tokens, hq + 2 * hkv, d).transpose(1, 2)
            q = apply_rope(qkv[:, :hq], self.cos, self.sin, start=start)
            k = apply_rope(qkv[:, hq:hq + hkv], self.cos, self.sin, start=start)
            v = qkv[:, hq + hkv:]
            cache.append(i, k, v)
            if start == 0:
                heads = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
            else:
                # A chunk after cached tokens attends its causal prefix straight from the pages.
                heads = paged_chunk_attention(q, *cache.pools(i), cache.block_table, ends,
                                              max_context_len=start + tokens)
            merged = heads.transpose(1, 2).reshape(batch * tokens, hq * d)
            x = torch.addmm(x.reshape(batch * tokens, -1), merged, w['self_attn.o_proj.weight'].t()).view(x.shape)
            x = self._mlp(x, w)
        cache.advance(tokens)
        return self._logits(x[:, -1])

    @torch.inference_mode()
    def decode(self, tokens: torch.Tensor, next_lens: torch.Tensor) -> torch.Tensor:
        """One new token per sequence ([B] ids) on the bound cache; logits [B, vocab].

        ``next_lens`` = the cache lengths + 1 (the new token included), a device
        tensor the caller keeps; the cache lengths are advanced by the caller.
        """
        batch = tokens.shape[0]
        hq, hkv, d = self.num_heads, self.num_kv_heads, self.head_dim
        x = F.embedding(tokens, self.embedding)
        for w, step in zip(self.layers, self._steps):
            h = rms_norm(x, w['input_layernorm.weight'], self.eps)
            qkv = F.linear(h, w['qkv'], w['qkv_bias']).view(batch, hq + 2 * hkv, d)
            heads = step(qkv[:, :hq], next_lens, key=qkv[:, hq:hq + hkv], value=qkv[:, hq + hkv:])
            x = torch.addmm(x, heads.view(batch, hq * d), w['self_attn.o_proj.weight'].t())
            x = self._mlp(x, w)
        return self._logits(x)


def prepare_model(weights, config) -> PreparedModel:
    """Bind a Qwen2 checkpoint (reference naming) for batched inference."""
    return PreparedModel(weights, config)
