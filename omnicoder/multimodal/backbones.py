"""Vision backbone family (reference src/omnicoder/modeling/multimodal/vision_encoder.py:6-423:
a ViT-tiny fallback plus timm / transformers backbones -- DINOv2, SigLIP, CLIP -- behind one
`VisionBackbone(backend)` that returns patch tokens and a pooled feature).

Backends (no download; weights are random unless a local directory is given):
  vit_tiny | vit_small | vit_base   ViT of the standard widths (192/3, 384/6, 768/12 heads,
                                    12 layers), class token pooled;
  dino_*                            same trunks, with 4 register tokens (dropped from the
                                    patch tokens) and mean-of-patches + class pooling;
  siglip_*                          no class token; attention-pooling head (a learned
                                    query attending over the patches);
  hf:<local dir>                    a transformers vision model loaded with
                                    local_files_only (last_hidden_state, pooler_output).
forward(images [B, 3, H, W]) -> (tokens [B, N, C], pooled [B, C]).
"""
from __future__ import annotations

import torch
import torch.nn as nn

WIDTHS = {"tiny": (192, 3), "small": (384, 6), "base": (768, 12)}


class _ViT(nn.Module):
    def __init__(self, dim: int, heads: int, depth: int, image_size: int, patch: int, cls: bool, registers: int):
        super().__init__()
        self.proj = nn.Conv2d(3, dim, patch, patch)
        self.n_patch = (image_size // patch) ** 2
        self.cls = nn.Parameter(torch.zeros(1, 1, dim)) if cls else None
        self.reg = nn.Parameter(torch.randn(1, registers, dim) * 0.02) if registers else None
        self.pos = nn.Parameter(torch.randn(1, self.n_patch + (1 if cls else 0), dim) * 0.02)
        layer = nn.TransformerEncoderLayer(dim, heads, 4 * dim, dropout=0.0, batch_first=True, norm_first=True,
                                           activation="gelu")
        self.blocks = nn.TransformerEncoder(layer, depth, enable_nested_tensor=False)
        self.norm = nn.LayerNorm(dim)

    def forward(self, img):
        x = self.proj(img).flatten(2).transpose(1, 2)
        B = x.shape[0]
        if self.cls is not None:
            x = torch.cat([self.cls.expand(B, -1, -1), x], 1)
        x = x + self.pos[:, :x.shape[1]]
        if self.reg is not None:
            x = torch.cat([x[:, :1], self.reg.expand(B, -1, -1), x[:, 1:]], 1)
        return self.norm(self.blocks(x))


class _AttnPool(nn.Module):
    def __init__(self, dim: int, heads: int):
        super().__init__()
        self.q = nn.Parameter(torch.randn(1, 1, dim) * 0.02)
        self.attn = nn.MultiheadAttention(dim, heads, batch_first=True)
        self.norm = nn.LayerNorm(dim)

    def forward(self, x):
        o, _ = self.attn(self.q.expand(x.shape[0], -1, -1), x, x)
        return self.norm(o[:, 0])


class VisionBackbone(nn.Module):
    def __init__(self, backend: str = "vit_tiny", image_size: int = 224, patch: int = 16, depth: int = 12):
        super().__init__()
        self.backend = backend
        self.hf = None
        if backend.startswith("hf:"):
            from transformers import AutoModel
            self.hf = AutoModel.from_pretrained(backend[3:], local_files_only=True)
            self.dim = int(getattr(self.hf.config, "hidden_size", 0) or self.hf.config.vision_config.hidden_size)
            return
        family, _, size = backend.partition("_")
        if family not in ("vit", "dino", "siglip") or size not in WIDTHS:
            raise ValueError(f"unknown vision backend {backend!r}")
        dim, heads = WIDTHS[size]
        self.family, self.dim = family, dim
        self.trunk = _ViT(dim, heads, depth, image_size, patch, cls=family != "siglip",
                          registers=4 if family == "dino" else 0)
        self.pool = _AttnPool(dim, heads) if family == "siglip" else None

    def forward(self, images: torch.Tensor):
        if self.hf is not None:
            out = self.hf(pixel_values=images)
            tok = out.last_hidden_state
            pooled = getattr(out, "pooler_output", None)
            return tok, (pooled if pooled is not None else tok.mean(1))
        x = self.trunk(images)
        if self.family == "vit":
            return x[:, 1:], x[:, 0]
        if self.family == "dino":
            patches = x[:, 5:]                      # class, 4 registers, patches
            return patches, 0.5 * (x[:, 0] + patches.mean(1))
        return x, self.pool(x)                      # siglip: no class token
