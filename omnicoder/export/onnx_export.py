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

Variants of the spec-family graph (reference onnx_export.py `--sfb_bias_input`,
`--head_verifier` / `--head_mtp`, `--prefill_multimodal`, `--emit_longctx_variants`,
`--kv_paged`, `--kvq`):
  * `logit_bias=True`: an extra input `logit_bias` [B, V] added to the logits (decoding
    add-ons such as SFB inject their token bias in-graph);
  * `heads=True`: extra outputs `verifier_logits` and `mtp_logits_j` from the same hidden
    state, when the model has those heads;
  * `MultimodalPrefillWrapper`: image pixels + prompt ids -> the fusion composer's
    composed embeddings -> logits and caches (the vision backbone is inside the graph);
  * `export_longctx_variants`: decode steps for 32k / 128k contexts (RoPE positions
    interpolated by target / trained length, the cache sized to the context);
  * sidecars: `*.kv_paging.json` (page length, pages per layer for a paged runtime) and
    `*.kvq.json` (u8 / nf4 group quantisation of the exported cache).
The export itself needs the `onnx` package (torch's exporter imports it); the
wrappers run and are tested without it (and trace under torch.export).
"""
from __future__ import annotations

import argparse

import torch
import torch.nn as nn


class DecodeStepWrapper(nn.Module):
    def __init__(self, model, logit_bias: bool = False, heads: bool = False):
        super().__init__()
        self.model = model
        self.compat = hasattr(model, "blocks") and hasattr(model.blocks[0], "step")
        if (logit_bias or heads) and self.compat:
            raise ValueError("logit_bias / head outputs are exported for the spec family")
        self.logit_bias, self.heads = logit_bias, heads
        if not self.compat and hasattr(model, "prepare_inference"):
            model.prepare_inference()                  # MLA: absorbed projections

    def head_names(self) -> list[str]:
        m = self.model
        if not self.heads:
            return []
        out = ["verifier_logits"] if getattr(m, "verifier", None) is not None else []
        return out + [f"mtp_logits_{j}" for j in range(len(getattr(m, "mtp_heads", [])))]

    def forward(self, input_ids, *cache):
        from ..ops.moe import static_shapes
        if not self.compat:
            bias = None
            if self.logit_bias:
                bias, cache = cache[-1], cache[:-1]
            with static_shapes():                      # routed experts without data-dependent shapes
                return self._spec_step(input_ids, *cache, bias=bias)
        if self.compat:
            L = len(self.model.blocks)
            past = [(cache[2 * i], cache[2 * i + 1]) for i in range(L)]
            out = self.model(input_ids, past_kv=past, use_cache=True)
            flat = [t for kv in out[1] for t in kv]
            return (out[0],) + tuple(flat)
        return self._spec_step(input_ids, *cache)

    def _spec_step(self, input_ids, position, *cache, bias=None, embeds=None):
        import math

        from ..models.lm import MLAttention
        from ..ops import linear_rope
        from ..ops.decode import decode_attention_torch
        m = self.model
        B, T = input_ids.shape if embeds is None else embeds.shape[:2]
        dev = (input_ids if embeds is None else embeds).device
        steps = position.reshape(1).long() + torch.arange(T, device=dev)                   # [T]
        pos = steps.reshape(1, T).expand(B, T)
        flat_pos = pos.reshape(-1)
        kv_len = (steps[-1] + 1).reshape(1).expand(B)
        h = m.embed[input_ids.reshape(-1)] if embeds is None else embeds.reshape(B * T, -1).to(m.embed.dtype)
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
        y = m.norm_f(h)
        logits = (y @ m.head_weight.t()).view(B, T, -1)
        if bias is not None:
            logits = logits + bias.reshape(B, 1, -1).to(logits.dtype)
        extra = []
        if self.heads:
            if getattr(m, "verifier", None) is not None:
                extra.append((y @ m.verifier.t()).view(B, T, -1))
            extra += [(y @ w.t()).view(B, T, -1) for w in getattr(m, "mtp_heads", [])]
        return (logits,) + tuple(new) + tuple(extra)


class MultimodalPrefillWrapper(nn.Module):
    """(pixel_values [B, 3, S, S], input_ids [B, T], position, caches) -> logits and caches of
    the composed sequence [image tokens with markers, text] (reference onnx_export.py
    `--prefill_multimodal`); the composer's vision backbone and projector run in the graph."""

    def __init__(self, model, composer):
        super().__init__()
        self.step = DecodeStepWrapper(model)
        if self.step.compat:
            raise ValueError("multimodal prefill is exported for the spec family")
        self.composer = composer

    def forward(self, pixel_values, input_ids, position, *cache):
        from ..ops.moe import static_shapes
        m = self.step.model
        emb, _ = self.composer.fuse_all(m.embed[input_ids], image=pixel_values)
        with static_shapes():
            return self.step._spec_step(input_ids, position, *cache, embeds=emb)


def io_names(n_layers: int, spec: bool = False, logit_bias: bool = False, head_names=()):
    ins = ["input_ids"] + (["position"] if spec else [])
    outs = ["logits"]
    for i in range(n_layers):
        ins += [f"k_lat_{i}", f"v_lat_{i}"]
        outs += [f"nk_lat_{i}", f"nv_lat_{i}"]
    if logit_bias:
        ins.append("logit_bias")
    return ins, outs + list(head_names)


def spec_cache_shapes(cfg, batch: int, max_len: int) -> list[tuple]:
    """(k_lat_i, v_lat_i) shapes of the spec family's exported cache, per layer."""
    if cfg.attn.kind == "mla":
        k = (batch, max_len, cfg.attn.kv_lora_rank + cfg.attn.qk_rope_dim)
        return [k, (batch, 1)] * cfg.n_layers          # v: a placeholder passed through
    kv = (batch, max_len, cfg.n_kv_heads, cfg.head_dim)
    return [kv, kv] * cfg.n_layers


def example_inputs(model, batch: int = 1, max_len: int = 256, tokens: int = 1, logit_bias: bool = False,
                   heads: bool = False):
    w = DecodeStepWrapper(model, logit_bias=logit_bias, heads=heads).eval()
    L = len(model.blocks)
    if w.compat:
        a = model.blocks[0].attn
        shape = (batch, a.n_heads, a.c.decode_window, a.dl)
        return w, (torch.zeros(batch, tokens, dtype=torch.long),) + tuple(torch.zeros(shape) for _ in range(2 * L))
    bias = (torch.zeros(batch, model.cfg.vocab_size),) if logit_bias else ()
    return w, (torch.zeros(batch, tokens, dtype=torch.long), torch.zeros((), dtype=torch.long)) + \
        tuple(torch.zeros(s) for s in spec_cache_shapes(model.cfg, batch, max_len)) + bias


def _require_onnx():
    try:
        import onnx  # noqa: F401
    except ImportError as e:
        raise RuntimeError("ONNX export needs the `onnx` package (not installed in this environment)") from e


def _export(model, path, batch, max_len, tokens, opset, logit_bias=False, heads=False):
    _require_onnx()
    w, args = example_inputs(model, batch, max_len, tokens, logit_bias, heads)
    ins, outs = io_names(len(model.blocks), spec=not w.compat, logit_bias=logit_bias, head_names=w.head_names())
    torch.onnx.export(w, args, path, input_names=ins, output_names=outs, opset_version=opset, dynamo=False)


def export_decode_step(model, path: str, batch: int = 1, max_len: int = 256, opset: int = 18,
                       logit_bias: bool = False, heads: bool = False) -> None:
    """One-token decode step graph (reference export/onnx_export.py:16-1764)."""
    _export(model, path, batch, max_len, 1, opset, logit_bias, heads)


def multimodal_example_inputs(model, composer, image_size: int, text_tokens: int, batch: int = 1,
                              max_len: int = 0):
    w = MultimodalPrefillWrapper(model, composer).eval()
    img = torch.zeros(batch, 3, image_size, image_size)
    ids = torch.zeros(batch, text_tokens, dtype=torch.long)
    with torch.no_grad():
        n = composer.fuse_all(model.embed[ids], image=img)[0].shape[1]     # composed length
    L = max_len or (n + 64)
    args = (img, ids, torch.zeros((), dtype=torch.long)) + \
        tuple(torch.zeros(s) for s in spec_cache_shapes(model.cfg, batch, L))
    return w, args


def export_multimodal_prefill(model, composer, path: str, image_size: int = 224, text_tokens: int = 32,
                              batch: int = 1, max_len: int = 0, opset: int = 18) -> None:
    _require_onnx()
    w, args = multimodal_example_inputs(model, composer, image_size, text_tokens, batch, max_len)
    ins, outs = io_names(len(model.blocks), spec=True)
    torch.onnx.export(w, args, path, input_names=["pixel_values"] + ins, output_names=outs, opset_version=opset,
                      dynamo=False)


def longctx_model(model, target_ctx: int):
    """A copy of the model's configuration for a `target_ctx` context: RoPE positions divided by
    target / trained length (position interpolation), the same weights."""
    import copy

    from ..config import get_rope_scale_for_target_ctx
    from ..ops.layers import RopeTable
    m = copy.copy(model)
    cfg = copy.deepcopy(model.cfg)
    scale = get_rope_scale_for_target_ctx(cfg.max_seq_len, target_ctx) * cfg.attn.rope_scale
    cfg.attn.rope_scale = scale
    cfg.max_seq_len = max(cfg.max_seq_len, target_ctx)
    m.cfg = cfg
    m.rope = RopeTable(model.rope.rot, cfg.max_seq_len, cfg.attn.rope_theta, scale)
    return m


def export_longctx_variants(model, out_prefix: str, ctxs=(32768, 131072), opset: int = 18) -> list[str]:
    """Decode-step graphs for long contexts (reference `--emit_longctx_variants`); the cache
    holds the full context (or the attention window when one is set)."""
    paths = []
    for ctx in ctxs:
        m = longctx_model(model, ctx)
        L = min(ctx, m.cfg.attn.window) if m.cfg.attn.window else ctx
        p = f"{out_prefix}_ctx{ctx // 1024}k.onnx"
        export_decode_step(m, p, max_len=L, opset=opset)
        paths.append(p)
    return paths


def write_sidecars(model, onnx_path: str, max_len: int, kv_page_len: int = 0, kvq: str = "none",
                   kvq_group: int = 64) -> list[str]:
    """JSON sidecars describing the exported cache for runtimes: paging and KV quantisation."""
    import json
    shapes = spec_cache_shapes(model.cfg, 1, max_len)
    base = onnx_path[:-5] if onnx_path.endswith(".onnx") else onnx_path
    out = []
    if kv_page_len:
        meta = {"page_len": kv_page_len, "max_len": max_len, "pages_per_layer": -(-max_len // kv_page_len),
                "n_layers": model.cfg.n_layers, "k_shape": list(shapes[0]), "v_shape": list(shapes[1]),
                "inputs": [f"k_lat_{i}" for i in range(model.cfg.n_layers)]}
        with open(base + ".kv_paging.json", "w") as f:
            json.dump(meta, f, indent=1)
        out.append(base + ".kv_paging.json")
    if kvq != "none":
        if kvq not in ("u8", "nf4"):
            raise ValueError("kvq: none | u8 | nf4")
        meta = {"scheme": kvq, "group": kvq_group, "bits": 8 if kvq == "u8" else 4,
                "per": "token x group of the last dim", "calibration": "runtime (per token)",
                "layers": model.cfg.n_layers}
        with open(base + ".kvq.json", "w") as f:
            json.dump(meta, f, indent=1)
        out.append(base + ".kvq.json")
    return out


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
    ap.add_argument("--opset", type=int, default=18)
    ap.add_argument("--sfb_bias_input", action="store_true", help="logit_bias input added to the logits")
    ap.add_argument("--heads", action="store_true", help="verifier / MTP head outputs")
    ap.add_argument("--emit_longctx_variants", action="store_true", help="also export 32k and 128k decode steps")
    ap.add_argument("--target_ctx", type=int, default=0, help="export for this context (RoPE interpolation)")
    ap.add_argument("--kv_page_len", type=int, default=0, help="write a KV paging sidecar with this page length")
    ap.add_argument("--kvq", default="none", choices=["none", "u8", "nf4"], help="write a KV quantisation sidecar")
    ap.add_argument("--kvq_group", type=int, default=64)
    a = ap.parse_args(argv)
    from ..inference.builders import load_model
    model, _ = load_model(a.ckpt, "cpu", dtype=torch.float32)
    model = model.eval()
    if a.target_ctx:
        model = longctx_model(model, a.target_ctx)
    export_decode_step(model, a.out, max_len=a.max_len, opset=a.opset, logit_bias=a.sfb_bias_input, heads=a.heads)
    write_sidecars(model, a.out, a.max_len, a.kv_page_len, a.kvq, a.kvq_group)
    if a.prefill:
        export_prefill(model, a.out.replace(".onnx", "") + "_prefill.onnx", a.prefill, max_len=a.max_len)
    if a.emit_longctx_variants:
        export_longctx_variants(model, a.out.replace(".onnx", ""), opset=a.opset)


if __name__ == "__main__":
    main()
