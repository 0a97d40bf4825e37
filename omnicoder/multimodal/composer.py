"""Modality composer (reference modeling/multimodal/fusion.py:64-681).

Builds one input sequence for the language model from text token embeddings
and other modalities, either as continuous features (projected to d_model and
wrapped in learned begin/end marker embeddings) or as discrete codes mapped into
the unified vocabulary (omnicoder.multimodal.vocab) and embedded by the LM's
own table.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .vocab import VocabSidecar


class MultimodalComposer(nn.Module):
    MODALITIES = ("image", "video", "audio")

    def __init__(self, d_model: int, feature_dims: dict | None = None, layout: VocabSidecar | None = None):
        super().__init__()
        dims = feature_dims or {"image": d_model, "video": d_model, "audio": d_model}
        self.proj = nn.ModuleDict({m: nn.Linear(d, d_model) for m, d in dims.items()})
        self.bos = nn.ParameterDict({m: nn.Parameter(torch.randn(d_model) * 0.02) for m in dims})
        self.eos = nn.ParameterDict({m: nn.Parameter(torch.randn(d_model) * 0.02) for m in dims})
        self.layout = layout or VocabSidecar.from_config()

    def fuse_features(self, text_emb: torch.Tensor, **features: torch.Tensor) -> torch.Tensor:
        """text_emb [B, T, D]; features[m] [B, n_m, dim_m] -> [B, sum, D]: modalities first, then text."""
        parts = []
        B = text_emb.shape[0]
        for m in self.MODALITIES:
            f = features.get(m)
            if f is None:
                continue
            parts += [self.bos[m].expand(B, 1, -1), self.proj[m](f), self.eos[m].expand(B, 1, -1)]
        return torch.cat(parts + [text_emb], 1)

    def map_codes(self, codes: torch.Tensor, modality: str) -> torch.Tensor:
        return codes + getattr(self.layout, f"{modality}_range")[0]

    def fuse_codes(self, text_ids: torch.Tensor, **codes: torch.Tensor) -> torch.Tensor:
        """Token ids of a unified-vocabulary sequence: mapped modality codes, then text."""
        parts = [self.map_codes(c, m) for m, c in codes.items() if c is not None]
        return torch.cat(parts + [text_ids], 1)
