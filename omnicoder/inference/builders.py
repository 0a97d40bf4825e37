"""Model builders and checkpoint loading for inference (reference
src/omnicoder/inference/generate.py:3279-3900: `maybe_load_checkpoint`,
`build_mobile_model`, `build_mobile_model_by_name`)."""
from __future__ import annotations

import torch

from ..config import ModelConfig, get_preset
from ..models.lm import OmniLM, build_model
from ..training.checkpoint import maybe_load_checkpoint


def build_mobile_model_by_name(name: str, rope_scale: float | None = None, rope_base: float | None = None,
                               multi_token: int = 1, mem_slots: int = 0, device="cpu", dtype=None) -> OmniLM:
    cfg = get_preset(name)
    if rope_scale is not None:
        cfg.attn.rope_scale = rope_scale
    if rope_base is not None:
        cfg.attn.rope_theta = rope_base
    cfg.mtp_heads = max(0, multi_token - 1)
    cfg.attn.mem_slots = mem_slots
    return build_model(cfg, device=device, dtype=dtype)


def build_mobile_model(cfg: ModelConfig, device="cpu", dtype=None) -> OmniLM:
    return build_model(cfg, device=device, dtype=dtype)


def load_model(ckpt: str, device="cpu", dtype=None, preset: str | None = None) -> tuple[OmniLM, dict]:
    """Build the model a checkpoint was trained with (its embedded config, else `preset`) and load it."""
    obj = torch.load(ckpt, map_location="cpu", weights_only=False)
    if isinstance(obj, dict) and "config" in obj:
        cfg = ModelConfig.from_dict(obj["config"])
    elif preset:
        cfg = get_preset(preset)
    else:
        raise ValueError(f"{ckpt} carries no model config; pass preset=")
    model = build_model(cfg, device=device, dtype=dtype)
    return model, maybe_load_checkpoint(model, ckpt)
