"""A CUDA graph keeps the split-KV workspace it captured.

The Python layer caches one split-KV workspace per (device, stream) and hands
a larger one to a call whose plan needs more. A graph that captured an
earlier call still writes into the earlier buffer, so that buffer must stay
allocated: if it were freed, the next capture (``torch.cuda.graph`` empties
the allocator's cache when it starts) could release it, and replaying the
graph would write into released memory.

The test checks the retention itself on the host before it replays anything,
then replays the graph after the cache has grown and been emptied, and
compares the output with the same call made eagerly and with the oracle.
"""
import pytest
import torch

from oracle import decode_float
from tests.golden.cases import make_inputs
from tests.helpers import as_float, assert_attention_close, to_numpy, workload_tensors

pytestmark = pytest.mark.gpu


def test_graph_keeps_its_workspace_when_a_later_call_needs_a_larger_one():
    from micro_vllm_b200 import cuda_attention, cuda_paged_cache

    inputs = make_inputs('qwen7b_bf16_small')
    t = workload_tensors(inputs)
    cuda_paged_cache.write_paged_kv(t['key_new'], t['value_new'], t['key_pool'], t['value_pool'],
                                    t['block_table'], positions=t['context_lens'], positions_are_end=True)
    stream = torch.cuda.Stream()
    key = (torch.cuda.current_device(), stream.cuda_stream)
    bound = int(inputs['context_lens'].max())
    out_eager = torch.empty_like(t['q'])
    out_graph = torch.empty_like(t['q'])

    def call(out, pages_per_split):
        cuda_attention.paged_decode_attention(t['q'], t['key_pool'], t['value_pool'], t['block_table'],
                                              t['context_lens'], max_context_len=bound, out=out,
                                              pages_per_split=pages_per_split)

    # Few splits: a small workspace, cached for this stream by the eager call.
    with torch.cuda.stream(stream):
        call(out_eager, 8)
    torch.cuda.synchronize()
    captured = cuda_attention._WORKSPACES[key].data_ptr()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        call(out_graph, 8)
    assert cuda_attention._WORKSPACES[key].data_ptr() == captured

    # Many splits on the same stream: the cache moves to a larger buffer.
    with torch.cuda.stream(stream):
        call(torch.empty_like(t['q']), 1)
    torch.cuda.synchronize()
    assert cuda_attention._WORKSPACES[key].data_ptr() != captured, 'expected a larger workspace'
    # The buffer the graph captured is still owned by the library.
    assert captured in {buf.data_ptr() for buf in cuda_attention._RETIRED_WORKSPACES}

    torch.cuda.empty_cache()
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out_graph.view(torch.int16), out_eager.view(torch.int16))
    expected = decode_float(inputs['q'], to_numpy(t['key_pool']), to_numpy(t['value_pool']),
                            inputs['block_table'], inputs['context_lens'], 128 ** -0.5, 'bfloat16')
    assert_attention_close(as_float(out_graph), expected, 'bfloat16')
    del graph
