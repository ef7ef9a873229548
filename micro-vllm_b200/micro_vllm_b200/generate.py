"""Batched greedy generation over a paged KV cache.

The reference's greedy loop decodes one request (src/micro_vllm/generate.py:82-107:
prefill once, then one token per forward, argmax, stop at EOS including it).
``greedy_decode`` runs the same loop for B requests of equal prompt length
at once: one batched prefill, then one decode step per new token for all
sequences, each step replayed from a CUDA graph (captured once; the decode
step's shapes never change). Per sequence, the result is what the reference
produces for that prompt alone.
"""
import torch

from .runtime import PreparedModel, prepare_model


def _eos_ids(eos_token_id, vocab_size):
    """generate.py:25-34: None or an empty sequence disables EOS stopping."""
    if eos_token_id is None:
        return ()
    ids = (eos_token_id,) if isinstance(eos_token_id, int) else eos_token_id
    if (not isinstance(ids, (tuple, list))
            or any(type(token) is not int or not 0 <= token < vocab_size for token in ids)):
        raise ValueError('EOS must be an integer ID, a list/tuple of valid IDs, or None')
    return tuple(ids)


class GreedyDecoder:
    """Prefill + graph-replayed decode steps for one batch; reusable across batches
    of the same shape (``run`` resets the cache)."""

    def __init__(self, model: PreparedModel, batch_size: int, capacity: int, *, page_size=16,
                 shuffle_seed=None, use_graph=True):
        self.model = model
        self.cache = model.allocate_cache(batch_size, capacity, page_size=page_size, shuffle_seed=shuffle_seed)
        model.bind(self.cache)
        self.use_graph = use_graph
        device = model.device
        self.tokens = torch.zeros(batch_size, dtype=torch.long, device=device)
        self.next_lens = torch.zeros(batch_size, dtype=torch.int32, device=device)
        self.stream = torch.cuda.Stream(device)
        self.graph = None

    def _step(self):
        """One decode step on the static buffers: advances lengths, writes the next tokens."""
        torch.add(self.cache.lengths, 1, out=self.next_lens)
        logits = self.model.decode(self.tokens, self.next_lens)
        self.cache.lengths.copy_(self.next_lens)
        self.tokens.copy_(logits.argmax(dim=-1))
        return logits

    def step(self):
        if not self.use_graph:
            self._step()
        elif self.graph is None:
            # The first step runs eagerly on the capture stream (allocating the
            # split-KV workspace there), the graph is captured from the second.
            self.stream.wait_stream(torch.cuda.current_stream(self.model.device))
            with torch.cuda.stream(self.stream):
                self._step()
            torch.cuda.current_stream(self.model.device).wait_stream(self.stream)
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                self._step()
        else:
            self.graph.replay()
        self.cache.note_advanced(1)

    @torch.inference_mode()
    def run(self, input_ids: torch.Tensor, max_new_tokens: int, eos_ids=()):
        self.cache.reset()
        logits = self.model.prefill(input_ids, self.cache)
        self.tokens.copy_(logits.argmax(dim=-1))
        generated = [self.tokens.clone()]
        finished = torch.zeros_like(self.tokens, dtype=torch.bool)
        eos = torch.tensor(eos_ids, device=self.tokens.device) if eos_ids else None
        for _ in range(max_new_tokens - 1):
            if eos is not None:
                finished |= torch.isin(generated[-1], eos)
                if bool(finished.all()):
                    break
            self.step()
            generated.append(self.tokens.clone())
        return torch.stack(generated, dim=1)


@torch.inference_mode()
def greedy_decode(weights, config, input_ids: torch.Tensor, max_new_tokens: int, *, eos_token_id=None,
                  page_size=16, use_graph=True):
    """Greedy tokens for B prompts of equal length: [B, new] int64, or a list of
    per-sequence tensors cut after their first EOS when ``eos_token_id`` is set.

    ``weights``: a checkpoint mapping in the reference's naming (with ``config``)
    or a ``PreparedModel``.
    """
    if type(max_new_tokens) is not int or max_new_tokens <= 0:
        raise ValueError('max_new_tokens must be a positive integer')
    if input_ids.ndim != 2 or input_ids.shape[1] == 0:
        raise ValueError('generation requires nonempty equal-length prompts [batch, tokens]')
    model = weights if isinstance(weights, PreparedModel) else prepare_model(weights, config)
    if input_ids.shape[1] + max_new_tokens - 1 > model.max_positions:
        raise ValueError('generation would require a forward beyond the configured context length')
    eos_ids = _eos_ids(eos_token_id, model.vocab)
    decoder = GreedyDecoder(model, input_ids.shape[0], input_ids.shape[1] + max_new_tokens - 1,
                            page_size=page_size, use_graph=use_graph)
    tokens = decoder.run(input_ids.to(model.device), max_new_tokens, eos_ids)
    if not eos_ids:
        return tokens
    out = []
    for row in tokens:
        hits = torch.isin(row, torch.tensor(eos_ids, device=row.device)).nonzero()
        out.append(row[:int(hits[0]) + 1] if len(hits) else row)
    return out
