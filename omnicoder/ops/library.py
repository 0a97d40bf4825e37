"""Dispatcher operators and backend registries.

`torch.ops.omnicoder.mla` / `torch.ops.omnicoder.matmul_int4` are registered by
the extension (C++ TORCH_LIBRARY, CUDA kernels for sm_100a, ATen on CPU): the
reference's native op namespace (src/omnicoder/modeling/kernels/dml_fused_attention.cpp:56-97,
loader omnicoder_dml_op.py) without the DirectML build.

MLA provider registry (reference src/omnicoder/modeling/kernels/mla_providers.py:30-184):
a provider is `fn(q, k, v, attn_mask, is_causal) -> out` over [BH, T, D] tensors.
Built in: "cuda" (the dispatcher op, tcgen05 flash attention where the shape allows)
and "cpu" (scaled_dot_product_attention in fp32).  The reference's "dml", "coreml"
and "nnapi" names resolve to "cpu" when no such runtime is present, as its own
fallbacks do.  The environment variable OMNICODER_MLA_PROVIDER picks the default.

`replace_linears_4bit` is the reference's bitsandbytes swap
(src/omnicoder/modeling/quant/providers.py:22-70) on this framework's own int4
weight-only layer (GEMV kernel for few rows, dequantise + GEMM otherwise).
"""
from __future__ import annotations

import os
from typing import Callable, Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _ext

MLAFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, Optional[torch.Tensor], bool], torch.Tensor]


def ops():
    """torch.ops.omnicoder, after the extension that registers it is loaded."""
    _ext.load()
    return torch.ops.omnicoder


def mla(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, attn_mask: torch.Tensor | None = None,
        is_causal: bool = False) -> torch.Tensor:
    return ops().mla(q, k, v, attn_mask, is_causal)


def matmul_int4(x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor | None = None,
                offset: float = 8.0) -> torch.Tensor:
    return ops().matmul_int4(x, packed, scale, zero, offset)


def _cpu_mla(q, k, v, attn_mask, is_causal):
    out = F.scaled_dot_product_attention(q.float(), k.float(), v.float(), attn_mask=attn_mask, is_causal=is_causal)
    return out.to(q.dtype)


_MLA: dict[str, MLAFn] = {"cpu": _cpu_mla, "cuda": mla}
_ALIASES = {"dml": "cpu", "coreml": "cpu", "nnapi": "cpu", "sdpa": "cpu"}


def register_mla_provider(name: str, fn: MLAFn) -> None:
    _MLA[name] = fn


def resolve_mla_provider(name: str | None = None, device: torch.device | str | None = None) -> MLAFn:
    """The provider called `name` (or OMNICODER_MLA_PROVIDER, or the device's default)."""
    name = name or os.environ.get("OMNICODER_MLA_PROVIDER") or None
    if name is None:
        name = "cuda" if torch.device(device or "cpu").type == "cuda" else "cpu"
    if name not in _MLA and name in _ALIASES:
        name = _ALIASES[name]
    if name not in _MLA:
        raise KeyError(f"unknown MLA provider {name!r}; known: {sorted(_MLA)}")
    return _MLA[name]


def replace_linears_4bit(module: nn.Module, skip: tuple = ("lm_head",)) -> int:
    """Swap every nn.Linear (names containing an entry of `skip` excepted) for Int4Linear;
    returns how many were replaced."""
    from ..quant.int4 import Int4Linear
    count = 0
    for name, mod in list(module.named_modules()):
        for cname, child in list(mod.named_children()):
            full = f"{name}.{cname}" if name else cname
            if isinstance(child, nn.Linear) and not any(s in full for s in skip):
                setattr(mod, cname, Int4Linear(child))
                count += 1
    return count
