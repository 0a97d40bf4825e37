"""CUDA-graph capture of incremental decode steps.

A decode step of the spec model is a few hundred small kernel launches (per
layer: norms, projections, rope, the KV-cache append, decode attention, the
router and the expert GEMMs); at batch 64 the GPU work per step is a few
milliseconds, so launch overhead and the gaps between launches are a large
share of it.  `GraphedStep` captures `model.forward_cached(ids, cache)` for a
fixed batch and number of new tokens once and replays it: the token ids are
copied into a static input buffer, the graph runs every kernel of the step, and
the cache lengths advance on the device exactly as in eager mode (positions,
visibility and cache rows are all read from `cache.lengths` on the device).

Limits: the cache, the model weights and the memory-row count
(`cache.n_mem`) must not change between capture and replay; a rollback
(speculative decoding) is a device copy into `cache.lengths` and needs no new
capture.
"""
from __future__ import annotations

import torch


class GraphedStep:
    def __init__(self, model, cache, tokens_per_step: int = 1, warmup: int = 2, return_hidden: bool = False):
        if not cache.device.type == "cuda":
            raise ValueError("GraphedStep needs a CUDA cache")
        self.model, self.cache = model, cache
        self.ids = torch.zeros(cache.batch, tokens_per_step, dtype=torch.long, device=cache.device)
        saved = cache.lengths.clone()
        side = torch.cuda.Stream(device=cache.device)
        side.wait_stream(torch.cuda.current_stream(cache.device))
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(warmup):          # first-call setup (attributes, tensor maps) outside the capture
                model.forward_cached(self.ids, cache, return_hidden=return_hidden)
                cache.rollback(saved)
        torch.cuda.current_stream(cache.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        self.hidden = None
        with torch.cuda.graph(self.graph), torch.no_grad():
            out = model.forward_cached(self.ids, cache, return_hidden=return_hidden)
        self.logits, self.hidden = out if return_hidden else (out, None)
        # capture records without executing: the cache is as it was before the warm-up
        cache.rollback(saved)

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        """ids [B, tokens_per_step] -> logits [B, tokens_per_step, V] (a view of the static output;
        the final hidden states, when captured, are in `self.hidden`)."""
        self.ids.copy_(ids)
        self.graph.replay()
        return self.logits
