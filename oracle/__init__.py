"""CPU oracle for the paged decode path.

TEST INFRASTRUCTURE ONLY. Nothing in the product package imports this
directory; only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
CPU-baseline leg use it, and only as the checker (or the timed CPU baseline),
never as the computation that is shipped or measured on the GPU.

``paged_attention`` restates micro-vllm's CPU reference path for one decode
step over a paged KV cache: ``PagedKVCache._gather_buffer`` /
``PagedKVCache.gather`` (src/micro_vllm/paged_kv_cache.py:178-193) followed by
``causal_attention`` (src/micro_vllm/attention.py:57-94), plus the fp64
per-head restatement the reference's CUDA tests use
(test/test_cuda_gqa.py:14-23).

``paged_append`` restates the cache write: ``PagedKVCache._append_cpu``
(src/micro_vllm/paged_kv_cache.py:151-161) and the native kernel's page
placement and invalid-ID skip (src/micro_vllm/csrc/paged_kv_cache.cu:18-41).

``rope`` restates the rotary embedding applied to q and K before the append
(``rotate_half`` / ``apply_rope``, src/micro_vllm/model.py:101-123).

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference's own
Python code on seeded inputs and commits the outputs under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks this oracle against them.
"""
from .dtypes import bf16_to_f32, f32_to_bf16, to_float32, from_float32, STORAGE_DTYPES
from .paged_append import append_tokens
from .rope import apply_rope
from .paged_attention import (
    decode_float,
    decode_fp64_per_head,
    decode_reference,
    gather_sequence,
)

__all__ = [
    'STORAGE_DTYPES', 'append_tokens', 'apply_rope', 'bf16_to_f32', 'decode_float',
    'decode_fp64_per_head', 'decode_reference', 'f32_to_bf16', 'from_float32',
    'gather_sequence', 'to_float32',
]
