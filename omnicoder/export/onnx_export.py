"""ONNX decode-step export (reference src/omnicoder/export/onnx_export.py:16-1764).

`DecodeStepWrapper` turns a model into a pure function of tensors with the
reference's I/O names: inputs `input_ids` [B, 1] and per layer `k_lat_i`,
`v_lat_i`; outputs `logits`, `nk_lat_i`, `nv_lat_i`.
  * compat family (OmniTransformer): the cache is the 16-slot latent window
    [B, H, 16, DL] per layer -- exactly the reference's decode-step graph.
  * spec family (OmniLM): the cache is the full K/V [B, L, Hk, D] (MLA: the
    compressed latent [B, L, r + dr] -- normalised latent and rotated rope key --
    with v_lat passed through unchanged) plus an extra `position` input; the T new
    entries are written at positions position .. position + T - 1.  MLA layers run
    in the absorbed form (query and output projections folded with the latent
    up-projections, attention over the latent rows).
`T > 1` tokens per call make the same function a prefill graph (`export_prefill`).
The export itself needs the `onnx` package (torch's exporter imports it); the
wrapper runs and is tested without it.
"""
from __future__ import annotations

import argparse

import torch
import torch.nn as nn


class DecodeStepWrapper(nn.Module):
    def __init__(self, model):
        super().__init__()
        self.model = model
        self.compat = hasattr(model, "blocks") and hasattr(model.blocks[0], "step")
        if not self.compat and hasattr(model, "prepare_inference"):
            model.prepare_inference()                  # MLA: absorbed projections

    def forward(self, input_ids, *cache):
        from ..ops.moe import static_shapes
        if not self.compat:
            with static_shapes():                      # routed experts without data-dependent shapes
                return self._spec_step(input_ids, *cache)
        if self.compat:
            L = len(self.model.blocks)
            past = [(cache[2 * i], cache[2 * i + 1]) for i in range(L)]
            out = self.model(input_ids, past_kv=past, use_cache=True)
            flat = [t for kv in out[1] for t in kv]
            return (out[0],) + tuple(flat)
        return self._spec_step(input_ids, *cache)

    def _spec_step(self, input_ids, position, *cache):
        import math

        from ..models.lm import MLAttention
        from ..ops import linear_rope
        from ..ops.decode import decode_attention_torch
        m = self.model
        B, T = input_ids.shape
        steps = position.reshape(1).long() + torch.arange(T, device=input_ids.device)     # [T]
        pos = steps.reshape(1, T).expand(B, T)
        flat_pos = pos.reshape(-1)
        kv_len = (steps[-1] + 1).reshape(1).expand(B)
        h = m.embed[input_ids.reshape(-1)]
        new = []
        for i, blk in enumerate(m.blocks):
            y = blk.attn_norm(h)
            k_c, v_c = cache[2 * i], cache[2 * i + 1]
            at = blk.attn
            if isinstance(at, MLAttention):
                r, dr, H = at.r, at.dr, at.H
                qa = linear_rope(y, at.wq_abs, m.rope, flat_pos, r + dr, H, off=r).view(B, T, H, r + dr)
                c, kr = at.latent(y, m.rope, flat_pos)
                k_c = k_c.index_copy(1, steps, torch.cat([c, kr], dim=-1).view(B, T, r + dr).to(k_c.dtype))
                o = decode_attention_torch(qa, k_c, None, pos, kv_len, scale=1.0 / math.sqrt(at.dn + dr),
                                           latent_v_dim=r)
                h = h + o.reshape(B * T, H * r) @ at.wo_abs.t()
            else:
                q, k, v, _ = at.qkv(y, m.rope, flat_pos)
                k_c = k_c.index_copy(1, steps, k.reshape(B, T, at.Hk, at.hd).to(k_c.dtype))
                v_c = v_c.index_copy(1, steps, v.reshape(B, T, at.Hk, at.hd).to(v_c.dtype))
                o = decode_attention_torch(q.reshape(B, T, at.H, at.hd), k_c, v_c, pos, kv_len)
                h = h + o.reshape(B * T, -1) @ at.wo.t()
            h = blk.ffn(blk.ffn_norm(h), h)[0]
            new += [k_c, v_c]
        logits = m.norm_f(h) @ m.head_weight.t()
        return (logits.view(B, T, -1),) + tuple(new)


def io_names(n_layers: int, spec: bool = False):
    ins = ["input_ids"] + (["position"] if spec else [])
    outs = ["logits"]
    for i in range(n_layers):
        ins += [f"k_lat_{i}", f"v_lat_{i}"]
        outs += [f"nk_lat_{i}", f"nv_lat_{i}"]
    return ins, outs


def spec_cache_shapes(cfg, batch: int, max_len: int) -> list[tuple]:
    """(k_lat_i, v_lat_i) shapes of the spec family's exported cache, per layer."""
    if cfg.attn.kind == "mla":
        k = (batch, max_len, cfg.attn.kv_lora_rank + cfg.attn.qk_rope_dim)
        return [k, (batch, 1)] * cfg.n_layers          # v: a placeholder passed through
    kv = (batch, max_len, cfg.n_kv_heads, cfg.head_dim)
    return [kv, kv] * cfg.n_layers


def example_inputs(model, batch: int = 1, max_len: int = 256, tokens: int = 1):
    w = DecodeStepWrapper(model).eval()
    L = len(model.blocks)
    if w.compat:
        a = model.blocks[0].attn
        shape = (batch, a.n_heads, a.c.decode_window, a.dl)
        return w, (torch.zeros(batch, tokens, dtype=torch.long),) + tuple(torch.zeros(shape) for _ in range(2 * L))
    return w, (torch.zeros(batch, tokens, dtype=torch.long), torch.zeros((), dtype=torch.long)) + \
        tuple(torch.zeros(s) for s in spec_cache_shapes(model.cfg, batch, max_len))


def _export(model, path, batch, max_len, tokens, opset):
    try:
        import onnx  # noqa: F401
    except ImportError as e:
        raise RuntimeError("ONNX export needs the `onnx` package (not installed in this environment)") from e
    w, args = example_inputs(model, batch, max_len, tokens)
    ins, outs = io_names(len(model.blocks), spec=not w.compat)
    torch.onnx.export(w, args, path, input_names=ins, output_names=outs, opset_version=opset, dynamo=False)


def export_decode_step(model, path: str, batch: int = 1, max_len: int = 256, opset: int = 18) -> None:
    """One-token decode step graph (reference export/onnx_export.py:16-1764)."""
    _export(model, path, batch, max_len, 1, opset)


def export_prefill(model, path: str, seq: int, batch: int = 1, max_len: int = 0, opset: int = 18) -> None:
    """Prefill graph of the spec family: `seq` tokens written at positions position .. + seq - 1,
    logits of every position (the same function as the decode step with T = seq)."""
    _export(model, path, batch, max_len or seq, seq, opset)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ckpt", required=True)
    ap.add_argument("--out", default="decode_step.onnx")
    ap.add_argument("--max_len", type=int, default=256)
    ap.add_argument("--prefill", type=int, default=0, help="also export a prefill graph of this many tokens")
    a = ap.parse_args(argv)
    from ..inference.builders import load_model
    model, _ = load_model(a.ckpt, "cpu", dtype=torch.float32)
    export_decode_step(model.eval(), a.out, max_len=a.max_len)
    if a.prefill:
        export_prefill(model.eval(), a.out.replace(".onnx", "") + "_prefill.onnx", a.prefill, max_len=a.max_len)


if __name__ == "__main__":
    main()
