"""Int4 weight-only linear layers.

Format (the reference's packer, src/omnicoder/modeling/quant/int4_linear.py:20-80):
per output row, symmetric scale = max|w| / 7, q = clamp(round(w / scale), -7, 7)
stored as the unsigned nibble q + 7; two nibbles per byte, element 2i in the
low nibble ("low_first"; "high_first" swaps them); rows zero-padded to a
multiple of 64 elements.  Value = (nibble - offset) * scale with offset 7.
The reference's kernel registry subtracts 8 instead of 7 (int4_kernels.py:33-60);
`matmul_int4(..., offset=8)` reproduces that behaviour, and the offset is
always explicit here.

CUDA: M <= 8 rows use the int4 GEMV kernel (weights read once, dequantised in
registers); larger M dequantise the weight to bf16 once and run the tcgen05
GEMM.  CPU: unpack + fp32 matmul (the oracle).
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.nn as nn

from ..ops import _ext

ALIGN = 64


def pack_int4(w: torch.Tensor, align: int = ALIGN, nibble_order: str = "low_first"):
    """w [N, K] -> (packed uint8 [N, Kp/2], scale fp32 [N], zero fp32 [N]) with Kp = K padded to `align`."""
    w = w.float()
    N, K = w.shape
    scale = (w.abs().amax(1) + 1e-8) / 7.0
    q = (torch.round(w / scale[:, None]).clamp(-7, 7) + 7).to(torch.uint8)
    Kp = (K + 1) // 2 * 2
    if align > 0:
        Kp = (Kp + align - 1) // align * align
    if Kp > K:
        q = torch.cat([q, torch.zeros(N, Kp - K, dtype=torch.uint8, device=q.device)], 1)
    lo, hi = q[:, 0::2], q[:, 1::2]
    packed = (lo | (hi << 4)) if nibble_order == "low_first" else ((lo << 4) | hi)
    return packed.contiguous(), scale, torch.zeros_like(scale)


def unpack_int4(packed: torch.Tensor, K: int, nibble_order: str = "low_first") -> torch.Tensor:
    a, b = packed & 0x0F, (packed >> 4) & 0x0F
    lo, hi = (a, b) if nibble_order == "low_first" else (b, a)
    q = torch.stack([lo, hi], -1).reshape(packed.shape[0], -1)
    return q[:, :K]


def dequant_int4(packed: torch.Tensor, scale: torch.Tensor, K: int, offset: float = 7.0, dtype=torch.float32,
                 nibble_order: str = "low_first") -> torch.Tensor:
    if packed.is_cuda and nibble_order == "low_first" and K % 8 == 0:
        return _ext.load().int4_dequant(packed, scale.float().contiguous(), K, offset).to(dtype)
    return ((unpack_int4(packed, K, nibble_order).float() - offset) * scale.float()[:, None]).to(dtype)


def _int4_cuda(x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, offset: float) -> torch.Tensor:
    C = _ext.load()
    x2 = x.reshape(-1, x.shape[-1]).to(torch.bfloat16).contiguous()
    K = x2.shape[1]
    if x2.shape[0] <= 8 and K % 8 == 0 and packed.shape[1] % 16 == 0:
        y = C.int4_gemv(x2, packed, scale.float().contiguous(), offset)
    else:
        from ..ops.gemm import mm_nt
        y = mm_nt(x2, C.int4_dequant(packed, scale.float().contiguous(), K, offset))
    return y.view(*x.shape[:-1], packed.shape[0])


def _int4_torch(x, packed, scale, offset):
    w = dequant_int4(packed, scale, x.shape[-1], offset)
    return x.float().matmul(w.t()).to(x.dtype)


_BACKENDS: dict[str, Callable] = {"cpu": _int4_torch, "cuda": _int4_cuda}


def register_int4_backend(name: str, fn: Callable) -> None:
    """Register a kernel `fn(x, packed, scale, offset) -> y` under `name` (reference int4_kernels.py:131)."""
    _BACKENDS[name] = fn


def matmul_int4(x: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor | None = None,
                offset: float = 8.0, backend: str | None = None) -> torch.Tensor:
    """y = x @ dequant(packed)^T.  Default offset 8 is the reference registry's convention;
    Int4Linear passes 7 (its packer's)."""
    name = backend or ("cuda" if x.is_cuda else "cpu")
    return _BACKENDS[name](x, packed, scale, offset)


class Int4Linear(nn.Module):
    """Drop-in weight-only int4 replacement of nn.Linear (reference quant/int4_linear.py:101)."""

    def __init__(self, linear: nn.Linear):
        super().__init__()
        self.in_features, self.out_features = linear.in_features, linear.out_features
        packed, scale, zero = pack_int4(linear.weight.data)
        self.register_buffer("packed_weight", packed)
        self.register_buffer("scale", scale)
        self.register_buffer("zero", zero)
        self.bias = None if linear.bias is None else nn.Parameter(linear.bias.data.clone(), requires_grad=False)

    def forward(self, x):
        y = matmul_int4(x, self.packed_weight, self.scale, self.zero, offset=7.0)
        return y if self.bias is None else y + self.bias.to(y.dtype)


def quantize_model_int4(model: nn.Module, skip: tuple = ("lm_head",)) -> nn.Module:
    """Replace every nn.Linear (except names containing an entry of `skip`) with Int4Linear."""
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            full = f"{name}.{cname}" if name else cname
            if isinstance(child, nn.Linear) and not any(s in full for s in skip):
                setattr(mod, cname, Int4Linear(child))
    return model
