"""``integration.install()`` rebinds micro-vllm's native names and restores them (CPU only)."""
from micro_vllm_b200 import cuda_attention, cuda_paged_cache, integration
from tests.reference_pkg import reference


def _bindings():
    model = reference('micro_vllm.model')
    ref_attention = reference('micro_vllm.cuda_attention')
    ref_cache = reference('micro_vllm.cuda_paged_cache')
    return (model.decode_attention_paged, ref_attention.decode_attention_paged,
            ref_attention.decode_attention_gqa, ref_cache._write_paged_kv)


def test_install_binds_this_package_and_restores_the_reference():
    before = _bindings()
    ours = (cuda_attention.decode_attention_paged, cuda_attention.decode_attention_paged,
            cuda_attention.decode_attention_gqa, cuda_paged_cache._write_paged_kv)
    assert all(a is not b for a, b in zip(before, ours))
    with integration.installed():
        assert all(a is b for a, b in zip(_bindings(), ours))
        with integration.installed():            # nested installs unwind in order
            assert all(a is b for a, b in zip(_bindings(), ours))
        assert all(a is b for a, b in zip(_bindings(), ours))
    assert all(a is b for a, b in zip(_bindings(), before))


def test_reference_model_checks_the_reference_cache_class_it_receives():
    """The drop-in's cache check accepts the reference's own PagedKVCache object."""
    PagedKVCache = reference('micro_vllm.paged_kv_cache').PagedKVCache
    cache = PagedKVCache.allocate(num_layers=1, num_kv_heads=1, num_pages=2, page_size=4, head_dim=8,
                                  dtype=cuda_attention.torch.float32, device='cpu')
    assert cuda_attention._is_paged_cache(cache)
    assert not cuda_attention._is_paged_cache(reference('micro_vllm.kv_cache').ContiguousKVCache.allocate(
        num_layers=1, batch_size=1, num_kv_heads=1, capacity=4, head_dim=8,
        dtype=cuda_attention.torch.float32, device='cpu'))
