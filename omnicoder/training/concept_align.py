"""Cross-modal alignment of the language model's concept head (reference
src/omnicoder/training/cross_modal_align.py:1-213: the LM's shared concept embedding is pulled
towards the frozen pre-aligned image and text embeddings of the same item).

  teacher (frozen):  z_img = PreAligner(image, vision(images)),  z_txt = PreAligner(text, TextEmbedder(ids))
  student:           z_c = ConceptLatentHead(LM hidden state at the last prompt position)   (unit norm)
  loss = InfoNCE(z_c, z_img) + InfoNCE(z_c, z_txt)                                 (temperature 0.07)
       + 0.5 * triplet(z_c, z_txt, z_txt_neg) + 0.5 * triplet(z_c, z_img, z_img_neg)  (cosine, margin 0.2)

InfoNCE is the symmetric cross entropy of the [B, B] similarity matrix / temperature against the
diagonal; triplet(a, p, n) = mean(max(0, (1 - a.p) - (1 - a.n) + margin)).  Negatives: the text
embeddings of prompts drawn from a negative list when one is given, otherwise the batch rotated by
one (every item is paired with a different item; a random permutation can leave an item paired with
itself, which makes its triplet term a constant).
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..models.heads import ConceptLatentHead


def info_nce(a: torch.Tensor, b: torch.Tensor, temperature: float = 0.07) -> torch.Tensor:
    logits = a.float() @ b.float().t() / max(temperature, 1e-6)
    target = torch.arange(a.shape[0], device=a.device)
    return 0.5 * (F.cross_entropy(logits, target) + F.cross_entropy(logits.t(), target))


def triplet(anchor: torch.Tensor, pos: torch.Tensor, neg: torch.Tensor, margin: float = 0.2) -> torch.Tensor:
    d_pos = 1.0 - (anchor * pos).sum(-1)
    d_neg = 1.0 - (anchor * neg).sum(-1)
    return (d_pos - d_neg + margin).clamp_min(0).mean()


class ConceptAligner:
    """Trains `head` (and optionally the LM) against a frozen teacher: `text` (ids -> features),
    `vision` (images -> features or (tokens, pooled)) and the `aligner` projecting both."""

    def __init__(self, lm, head: ConceptLatentHead, text: nn.Module, vision: nn.Module, aligner: nn.Module,
                 lr: float = 1e-3, train_lm: bool = False, temperature: float = 0.07, margin: float = 0.2):
        self.lm, self.head, self.text, self.vision, self.aligner = lm, head, text, vision, aligner
        self.train_lm, self.temperature, self.margin = train_lm, temperature, margin
        for m in (text, vision, aligner):
            m.requires_grad_(False)
        params = list(head.parameters()) + ([p for p in lm.parameters() if p.requires_grad] if train_lm else [])
        self.opt = torch.optim.AdamW(params, lr=lr)

    @torch.no_grad()
    def teacher(self, images: torch.Tensor, ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        v = self.vision(images)
        if isinstance(v, tuple):
            v = v[1] if v[1] is not None else v[0].mean(1)
        return self.aligner("image", v).float(), self.aligner("text", self.text(ids)).float()

    def concept(self, ids: torch.Tensor) -> torch.Tensor:
        ctx = torch.enable_grad() if self.train_lm else torch.no_grad()
        with ctx:
            y, _ = self.lm.hidden(ids)
        h = y.view(ids.shape[0], ids.shape[1], -1)
        return self.head(h.float()).float()

    def loss(self, images: torch.Tensor, ids: torch.Tensor, neg_ids: torch.Tensor | None = None):
        z_img, z_txt = self.teacher(images, ids)
        z_c = self.concept(ids)
        loss = info_nce(z_c, z_img, self.temperature) + info_nce(z_c, z_txt, self.temperature)
        if neg_ids is not None:
            with torch.no_grad():
                z_neg = self.aligner("text", self.text(neg_ids)).float()
        else:
            z_neg = z_txt.roll(1, 0)
        t_txt = triplet(z_c, z_txt, z_neg, self.margin)
        t_img = triplet(z_c, z_img, z_img.roll(1, 0), self.margin)
        loss = loss + 0.5 * t_txt + 0.5 * t_img
        return loss, {"loss": float(loss.detach()), "triplet_text": float(t_txt.detach()),
                      "triplet_image": float(t_img.detach())}

    def step(self, images: torch.Tensor, ids: torch.Tensor, neg_ids: torch.Tensor | None = None) -> dict:
        loss, parts = self.loss(images, ids, neg_ids)
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        self.opt.step()
        return parts

    @torch.no_grad()
    def retrieval_accuracy(self, images: torch.Tensor, ids: torch.Tensor) -> float:
        """Fraction of items whose concept embedding is closest to its own image embedding."""
        z_img, _ = self.teacher(images, ids)
        z_c = self.concept(ids)
        return float(((z_c @ z_img.t()).argmax(1) == torch.arange(len(ids), device=ids.device)).float().mean())


def _pad(rows: list[list[int]], device) -> torch.Tensor:
    L = max(1, max(len(r) for r in rows))
    return torch.tensor([r + [0] * (L - len(r)) for r in rows], dtype=torch.long, device=device)


def main(argv=None):
    from ..config import get_preset
    from ..models.lm import build_model
    from ..multimodal.aligner import PreAligner
    from ..multimodal.backbones import VisionBackbone
    from .pre_align import TextEmbedder
    from .tokenizer import get_tokenizer
    ap = argparse.ArgumentParser(description="align the LM concept head with pre-aligned image / text embeddings")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--pre_align_ckpt", default="", help="aligner + text embedder saved by the pre-alignment run")
    ap.add_argument("--vision", default="vit_tiny")
    ap.add_argument("--image_size", type=int, default=32)
    ap.add_argument("--embed_dim", type=int, default=192)
    ap.add_argument("--shared", type=int, default=128)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--neg_text", action="store_true", help="negatives from a fixed list of unrelated prompts")
    ap.add_argument("--out", default="weights/concept_head.pt")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dev = torch.device(a.device)
    lm = build_model(get_preset(a.preset), device=dev, dtype=torch.float32, seed=0).eval()
    tok = get_tokenizer(lm.cfg.vocab_size)
    vision = VisionBackbone(a.vision, image_size=a.image_size, depth=2)
    text = TextEmbedder(32000, a.embed_dim)
    aligner = PreAligner({"text": a.embed_dim, "image": vision.dim}, a.shared)
    if a.pre_align_ckpt:
        ck = torch.load(a.pre_align_ckpt, map_location="cpu", weights_only=True)
        aligner.load_state_dict(ck["aligner"], strict=False)
        text.load_state_dict(ck["text"])
    head = ConceptLatentHead(lm.cfg.d_model, a.shared).to(dev)
    tr = ConceptAligner(lm, head, text.to(dev), vision.to(dev).eval(), aligner.to(dev), a.lr)
    g = torch.Generator().manual_seed(0)
    colors = torch.rand(16, 3, generator=g)
    caps = [f"a {['red', 'green', 'blue', 'grey'][i % 4]} square number {i}" for i in range(16)]
    negs = ["a recipe for bread", "the stock market fell", "a poem about rain", "quarterly tax forms"]
    log = []
    for _ in range(a.steps):
        idx = torch.randperm(16, generator=g)[:a.batch]
        imgs = colors[idx][:, :, None, None].expand(-1, -1, a.image_size, a.image_size).contiguous().to(dev)
        ids = _pad([tok.encode(caps[int(i)]) for i in idx], dev)
        neg = _pad([tok.encode(negs[int(i) % len(negs)]) for i in idx], dev) if a.neg_text else None
        log.append(tr.step(imgs, ids, neg))
    torch.save({"concept_head": head.state_dict()}, a.out)
    print(json.dumps({"steps": a.steps, "first": log[0], "last": log[-1], "out": a.out}))
    return 0


if __name__ == "__main__":
    main()
