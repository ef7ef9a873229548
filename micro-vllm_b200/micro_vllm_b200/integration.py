"""Route an installed micro-vllm's native decode path to this package.

micro-vllm reaches its CUDA decode path through module-level names that its
own code looks up when it runs, so rebinding them is the whole integration; no
reference source changes:

* ``micro_vllm.model.decode_attention_paged`` -- imported by name into the
  model module (src/micro_vllm/model.py:12) and called by
  ``_attention_with_cache`` for a paged cache in CUDA mode (model.py:175-177);
* ``micro_vllm.cuda_attention.decode_attention_paged`` -- the public name of
  the same function (src/micro_vllm/cuda_attention.py:116-135);
* ``micro_vllm.cuda_attention.decode_attention_gqa`` -- the contiguous-cache
  decode, imported at call time by ``attention_forward``
  (src/micro_vllm/attention_backend.py:80-84);
* ``micro_vllm.cuda_paged_cache._write_paged_kv`` -- the cache write, imported
  at call time by ``PagedKVCache.append`` (src/micro_vllm/paged_kv_cache.py:163-172).

These are the names micro-vllm's own tests patch to observe its native path
(test/test_paged_forward.py:131-134). After ``install()``, micro-vllm's model
code, its ``PagedKVCache`` and its generation loop run this package's sm_100a
kernels; the reference's JIT-built extensions are never loaded.
"""
import contextlib
import importlib

# (micro-vllm module, name there, this package's module, name here)
BINDINGS = (
    ('micro_vllm.model', 'decode_attention_paged', 'cuda_attention', 'decode_attention_paged'),
    ('micro_vllm.cuda_attention', 'decode_attention_paged', 'cuda_attention', 'decode_attention_paged'),
    ('micro_vllm.cuda_attention', 'decode_attention_gqa', 'cuda_attention', 'decode_attention_gqa'),
    ('micro_vllm.cuda_paged_cache', '_write_paged_kv', 'cuda_paged_cache', '_write_paged_kv'),
)


def install():
    """Rebind micro-vllm's native decode names to this package's functions.

    micro-vllm must be importable. Returns a callable that restores the
    previous bindings (in reverse order, so nested installs unwind cleanly).
    """
    saved = []
    for module_name, name, ours_module, ours_name in BINDINGS:
        module = importlib.import_module(module_name)
        ours = getattr(importlib.import_module(f'{__package__}.{ours_module}'), ours_name)
        saved.append((module, name, getattr(module, name)))
        setattr(module, name, ours)

    def restore():
        for module, name, previous in reversed(saved):
            setattr(module, name, previous)

    return restore


@contextlib.contextmanager
def installed():
    """``install()`` for the duration of a ``with`` block."""
    restore = install()
    try:
        yield
    finally:
        restore()
