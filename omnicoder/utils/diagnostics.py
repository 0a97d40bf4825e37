"""Expert-load diagnostics for MoE models (the reference computes load statistics inside
its MoE layer and discards them, src/omnicoder/modeling/moe_layer.py:836-858).

`expert_load(model, ids)` runs one no-grad forward with a pre-hook on every routed
FFN, applies that layer's router to the layer's input (softmax, top-k) and counts the
chosen experts on the device.  Returns per-layer counts [L, E] and summary figures:
the coefficient of variation of each layer's load (0 = perfectly even) and the
share of the busiest expert.
"""
from __future__ import annotations

import torch


@torch.no_grad()
def expert_load(model, ids: torch.Tensor) -> dict:
    k = model.cfg.moe.top_k
    counts, hooks = [], []

    def hook(mod, args):
        x = args[0].reshape(-1, args[0].shape[-1]).float()
        idx = (x @ mod.router.float().t()).topk(k, dim=-1).indices
        counts.append(torch.bincount(idx.reshape(-1), minlength=mod.router.shape[0]))

    for blk in model.blocks:
        ffn = getattr(blk, "ffn", None)
        if ffn is not None and hasattr(ffn, "router"):
            hooks.append(ffn.register_forward_pre_hook(hook))
    try:
        model.hidden(ids)
    finally:
        for h in hooks:
            h.remove()
    if not counts:
        return {"counts": None, "cv": [], "max_share": []}
    c = torch.stack(counts).float()                         # [L, E]
    cv = (c.std(1, unbiased=False) / c.mean(1).clamp_min(1e-9)).tolist()
    share = (c.max(1).values / c.sum(1).clamp_min(1)).tolist()
    return {"counts": c.long().cpu(), "cv": cv, "max_share": share}
