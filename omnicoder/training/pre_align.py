"""Pre-alignment of the modality encoders into one embedding space (reference
src/omnicoder/training/pre_align.py:55-140: a small text embedder and the vision / audio / video
backbones projected by a PreAligner and trained with symmetric InfoNCE, text-image at weight 1 and
audio-text, video-text at 0.5 when those modalities are present).

A batch holds captions and any of images [B, 3, S, S], audio waves [B, samples] and video clips
[B, T, 3, S, S] describing the same items; the aligner is what the fusion composer's projectors and
the cross-modal verifier start from.
"""
from __future__ import annotations

import argparse
import json
import math

import torch
import torch.nn as nn

from ..multimodal.aligner import PreAligner, clip_loss


class TextEmbedder(nn.Module):
    """Mean of learned token embeddings over the non-padding tokens (id 0 is padding)."""

    def __init__(self, vocab_size: int, dim: int):
        super().__init__()
        self.emb = nn.Embedding(vocab_size, dim)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        m = (ids != 0).float()[..., None]
        return (self.emb(ids) * m).sum(1) / m.sum(1).clamp_min(1.0)


class PreAlignTrainer:
    def __init__(self, text: TextEmbedder, encoders: dict, shared: int = 256, lr: float = 1e-3,
                 weights: dict | None = None):
        self.text, self.enc = text, nn.ModuleDict(encoders)
        dims = {"text": text.emb.embedding_dim}
        for k, e in encoders.items():
            d = getattr(e, "dim", None) or getattr(e, "out_dim", None)
            if d is None and hasattr(e, "proj"):          # projection-headed encoders (mel front end)
                d = e.proj.out_features
            dims[k] = d
        self.align = PreAligner(dims, shared)
        self.logit_scale = nn.Parameter(torch.tensor(math.log(1 / 0.07)))
        self.weights = {"image": 1.0, "audio": 0.5, "video": 0.5, **(weights or {})}
        params = list(text.parameters()) + list(self.enc.parameters()) + list(self.align.parameters()) + \
            [self.logit_scale]
        self.opt = torch.optim.AdamW(params, lr=lr)

    def _feat(self, kind: str, x: torch.Tensor) -> torch.Tensor:
        out = self.enc[kind](x)
        if isinstance(out, tuple):
            out = out[1] if kind == "image" else out[0]     # vision: pooled; video: per-frame features
        return out

    def loss(self, ids: torch.Tensor, **media) -> tuple[torch.Tensor, dict]:
        t = self.align("text", self.text(ids))
        total, parts = 0.0, {}
        for kind, x in media.items():
            if x is None:
                continue
            m = self.align(kind, self._feat(kind, x))
            l_k = clip_loss(t, m, self.logit_scale)
            total = total + self.weights.get(kind, 1.0) * l_k
            parts[kind] = float(l_k.detach())
        return total, parts

    def step(self, ids: torch.Tensor, **media) -> dict:
        loss, parts = self.loss(ids, **media)
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        self.opt.step()
        return parts


def main(argv=None):
    from ..multimodal.backbones import VisionBackbone
    from ..multimodal.encoders import MelFrontend
    from .tokenizer import get_tokenizer
    ap = argparse.ArgumentParser(description="modality pre-alignment (InfoNCE)")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--image_size", type=int, default=32)
    ap.add_argument("--vision", default="vit_tiny")
    ap.add_argument("--embed_dim", type=int, default=192)
    ap.add_argument("--shared", type=int, default=128)
    ap.add_argument("--audio", action="store_true", help="also align synthetic audio tones")
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--out", default="weights/pre_align.pt")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dev = torch.device(a.device)
    tok = get_tokenizer(32000)
    enc = {"image": VisionBackbone(a.vision, image_size=a.image_size, depth=2)}
    if a.audio:
        enc["audio"] = MelFrontend(out_dim=a.embed_dim)
    tr = PreAlignTrainer(TextEmbedder(32000, a.embed_dim), enc, a.shared, a.lr)
    for m in (tr.text, tr.enc, tr.align):
        m.to(dev)
    tr.logit_scale.data = tr.logit_scale.data.to(dev)
    g = torch.Generator().manual_seed(0)
    colors = torch.rand(16, 3, generator=g)
    caps = [f"a {['red', 'green', 'blue', 'grey'][i % 4]} square number {i}" for i in range(16)]
    log = []
    for _ in range(a.steps):
        idx = torch.randperm(16, generator=g)[:a.batch]
        imgs = colors[idx][:, :, None, None].expand(-1, -1, a.image_size, a.image_size).contiguous().to(dev)
        enc_ids = [tok.encode(caps[int(i)]) for i in idx]
        L = max(len(e) for e in enc_ids)
        ids = torch.tensor([e + [0] * (L - len(e)) for e in enc_ids], device=dev)
        media = {"image": imgs}
        if a.audio:
            tt = torch.arange(4000, device=dev) / 16000.0
            media["audio"] = torch.stack([torch.sin(2 * math.pi * (200 + 50 * float(i)) * tt) for i in idx])
        log.append(tr.step(ids, **media))
    torch.save({"aligner": tr.align.state_dict(), "text": tr.text.state_dict()}, a.out)
    print(json.dumps({"steps": a.steps, "first": log[0], "last": log[-1], "out": a.out}))
    return 0


if __name__ == "__main__":
    main()
