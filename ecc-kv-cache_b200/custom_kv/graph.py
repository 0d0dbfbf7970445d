"""Greedy decoding with each step one CUDA-graph replay.

The reference decodes eagerly (custom_kv/patch.py:100, one Python pass over
every layer per token); at batch 1 that step is bound by host-side work.  Here
one decode step of a transformers causal LM -- the model's forward for one
token with the ErrorCorrectedCache (append + fused decode per layer, lengths
in device memory), the argmax and the advance of every position counter -- is
recorded once and replayed per token.
"""
from __future__ import annotations

import torch

from .cache import ErrorCorrectedCache


class GraphDecoder:
    """Greedy decode steps of ``model`` over ``cache`` as CUDA-graph replays.

    ``first_token`` [B, 1] (int64, on the GPU) is the token that follows the
    ``cache``'s current content (typically the argmax of the prefill logits).
    The SDPA patch of ``cache`` must be active (``ecc_cache`` or
    ``patch_model``) while the decoder is made, and the batch must be unpadded
    (replays do not read an attention mask).  Each ``step()`` feeds the
    current token, appends its K/V to every layer, and returns the next token
    (a device tensor the next replay overwrites).  The cache's host-side
    lengths are not advanced by replays; ``sync_host_lengths()`` reads them back.
    """

    def __init__(self, model, cache: ErrorCorrectedCache, first_token: torch.Tensor):
        if not isinstance(cache, ErrorCorrectedCache):
            raise TypeError("GraphDecoder needs an ErrorCorrectedCache")
        if cache._last_window is not None:
            # replays do not read the attention mask (it is not a graph input)
            raise RuntimeError("GraphDecoder serves unpadded batches: the last forward pass had an attention mask "
                               "that excludes cached tokens")
        self.model = model
        self.cache = cache
        dev = cache._device
        self.n0 = cache.get_seq_length(0)
        cache.enable_device_lengths()
        B = first_token.shape[0]
        self.ids = first_token.reshape(B, 1).to(device=dev, dtype=torch.long).clone()
        self.cache_position = torch.full((1,), self.n0, dtype=torch.long, device=dev)
        self.position_ids = torch.full((B, 1), self.n0, dtype=torch.long, device=dev)
        fills = list(cache._layer_fill)
        # one eager step off the capture: workspaces, tensor maps, kernel
        # attributes and the allocator's blocks exist before recording; its
        # token and the counters are then put back
        first = self.ids.clone()
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            self._step()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self._rewind(first, fills)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.next_token = self._step()
        self._rewind(first, fills)
        self.steps = 0

    def _rewind(self, first: torch.Tensor, fills) -> None:
        self.ids.copy_(first)
        self.cache_position.fill_(self.n0)
        self.position_ids.fill_(self.n0)
        self.cache.set_device_lengths(self.n0)
        self.cache._layer_fill[:] = fills

    def _step(self) -> torch.Tensor:
        out = self.model(input_ids=self.ids, position_ids=self.position_ids, cache_position=self.cache_position,
                         past_key_values=self.cache, use_cache=True)
        self.logits = out.logits[:, -1]
        nxt = self.logits.argmax(-1, keepdim=True)
        self.ids.copy_(nxt)
        self.cache_position.add_(1)
        self.position_ids.add_(1)
        self.cache.advance_device_lengths()
        return nxt

    def step(self) -> torch.Tensor:
        """One decode step; returns the next token [B, 1] (device tensor)."""
        if self.n0 + self.steps + 1 > self.cache.get_max_cache_shape():
            raise RuntimeError("cache full")
        self.graph.replay()
        self.steps += 1
        return self.next_token

    def sync_host_lengths(self) -> int:
        """Copy the device-side length back into the cache's host bookkeeping
        (synchronises); returns the number of cached tokens."""
        n = int(self.cache._pos_dev.item())
        self.cache._layer_fill[:] = [n] * len(self.cache._layer_fill)
        self.cache._seen_tokens = n
        return n
