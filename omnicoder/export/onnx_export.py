"""ONNX decode-step export (reference src/omnicoder/export/onnx_export.py:16-1764).

`DecodeStepWrapper` turns a model into a pure function of tensors with the
reference's I/O names: inputs `input_ids` [B, 1] and per layer `k_lat_i`,
`v_lat_i`; outputs `logits`, `nk_lat_i`, `nv_lat_i`.
  * compat family (OmniTransformer): the cache is the 16-slot latent window
    [B, H, 16, DL] per layer -- exactly the reference's decode-step graph.
  * spec family (OmniLM): the cache is the full K/V [B, L, Hk, D] (MLA: the
    latent [B, L, r + dr] with v_lat an empty placeholder) plus an extra
    `position` input; the new entry is written at `position`.
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

    def forward(self, input_ids, *cache):
        if self.compat:
            L = len(self.model.blocks)
            past = [(cache[2 * i], cache[2 * i + 1]) for i in range(L)]
            out = self.model(input_ids, past_kv=past, use_cache=True)
            flat = [t for kv in out[1] for t in kv]
            return (out[0],) + tuple(flat)
        return self._spec_step(input_ids, *cache)

    def _spec_step(self, input_ids, position, *cache):
        from ..ops.decode import decode_attention_torch
        m = self.model
        B = input_ids.shape[0]
        pos = position.reshape(1, 1).expand(B, 1).long()
        h = m.embed[input_ids.reshape(-1)]
        new = []
        for i, blk in enumerate(m.blocks):
            y = blk.attn_norm(h)
            k_c, v_c = cache[2 * i], cache[2 * i + 1]
            at = blk.attn
            if hasattr(at, "wq_abs"):
                raise NotImplementedError("MLA decode-step export: use the compat family or the GQA spec family")
            q, k, v, _ = at.qkv(y, m.rope, pos.reshape(-1))
            k_c = k_c.index_copy(1, pos[0], k.reshape(B, 1, at.Hk, at.hd))
            v_c = v_c.index_copy(1, pos[0], v.reshape(B, 1, at.Hk, at.hd))
            o = decode_attention_torch(q.reshape(B, 1, at.H, at.hd), k_c, v_c, pos, pos[:, 0] + 1)
            h = h + o.reshape(B, -1) @ at.wo.t()
            h = blk.ffn(blk.ffn_norm(h), h)[0]
            new += [k_c, v_c]
        logits = m.norm_f(h) @ m.head_weight.t()
        return (logits.view(B, 1, -1),) + tuple(new)


def io_names(n_layers: int, spec: bool = False):
    ins = ["input_ids"] + (["position"] if spec else [])
    outs = ["logits"]
    for i in range(n_layers):
        ins += [f"k_lat_{i}", f"v_lat_{i}"]
        outs += [f"nk_lat_{i}", f"nv_lat_{i}"]
    return ins, outs


def export_decode_step(model, path: str, batch: int = 1, max_len: int = 256, opset: int = 18) -> None:
    try:
        import onnx  # noqa: F401
    except ImportError as e:
        raise RuntimeError("ONNX export needs the `onnx` package (not installed in this environment)") from e
    w = DecodeStepWrapper(model).eval()
    L = len(model.blocks)
    if w.compat:
        a = model.blocks[0].attn
        shape = (batch, a.n_heads, a.c.decode_window, a.dl)
        args = (torch.zeros(batch, 1, dtype=torch.long),) + tuple(torch.zeros(shape) for _ in range(2 * L))
    else:
        c = model.cfg
        shape = (batch, max_len, c.n_kv_heads, c.head_dim)
        args = (torch.zeros(batch, 1, dtype=torch.long), torch.zeros((), dtype=torch.long)) + \
            tuple(torch.zeros(shape) for _ in range(2 * L))
    ins, outs = io_names(L, spec=not w.compat)
    torch.onnx.export(w, args, path, input_names=ins, output_names=outs, opset_version=opset, dynamo=False)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ckpt", required=True)
    ap.add_argument("--out", default="decode_step.onnx")
    ap.add_argument("--max_len", type=int, default=256)
    a = ap.parse_args(argv)
    from ..inference.builders import load_model
    model, _ = load_model(a.ckpt, "cpu", dtype=torch.float32)
    export_decode_step(model.eval(), a.out, max_len=a.max_len)


if __name__ == "__main__":
    main()
