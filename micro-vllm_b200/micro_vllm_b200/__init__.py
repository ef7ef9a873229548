"""B200-native paged decode path for micro-vllm.

Hand-written sm_100a CUDA kernels for paged GQA decode attention (split-KV,
TMA page staging, tensor-core tiles) and the paged KV append, behind a C ABI
(libmvdecode.so, include/mvdecode.h) and host wrappers that keep micro-vllm's
own function names, arguments and errors:

    cuda_attention.decode_attention_paged        <- micro_vllm.cuda_attention
    cuda_attention.decode_attention_gqa          <- micro_vllm.cuda_attention
    cuda_paged_cache._write_paged_kv             <- micro_vllm.cuda_paged_cache

``integration.install()`` rebinds those names inside an installed micro-vllm,
so its own model code and its own ``PagedKVCache`` run on these kernels.

Beyond the reference: batched forms (``paged_decode_attention``,
``write_paged_kv``, and the one-call append + attend step
``paged_decode_with_append``) over one shared page pool, a batched cache and
runtime (``paged_kv_cache.BatchedPagedKVCache``, ``runtime``, ``generate``),
and KV-head sharding across GPUs (``sharding``).
"""
__version__ = '0.1.0'
