"""Tensor-level wrappers of the tcgen05 GEMM.

Conventions (all bf16, fp32 accumulation):
  ``mm_nt(a, b)``  = a @ b.T   a [M,K], b [N,K]     (forward of a linear layer)
  ``mm_nn(a, b)``  = a @ b     a [M,K], b [K,N]     (input gradient)
  ``mm_tn(a, b)``  = a.T @ b   a [K,M], b [K,N]     (weight gradient)
On CPU the same functions run torch.matmul; that path is the fp32 oracle.
"""
from __future__ import annotations

import os

import torch

from . import _ext

EPI_BF16, EPI_F32, EPI_ACC_F32, EPI_ADD, EPI_SWIGLU, EPI_SWIGLU_BWD = range(6)

# Plain few-row GEMMs (decode-step projections: bf16 out, optional residual, no fused epilogue) with
# at most this many rows go to the library GEMM (cuBLAS through torch.mm / addmm); 0 keeps them on
# the few-row tcgen05 kernel.  At 64 rows the library is faster on these dense weight-streaming
# shapes (batch-64 decode step 8.24 -> 7.5-7.8 ms); the packed per-expert GEMMs and the fused
# SwiGLU projections stay on the tcgen05 kernels.  Read once at import.
FEW_ROW_LIBRARY_MAX = int(os.environ.get("OMNI_FEW_ROW_LIBRARY", "64"))


def _c2d(t: torch.Tensor) -> torch.Tensor:
    return t if (t.dim() == 2 and t.stride(-1) == 1) else t.reshape(-1, t.shape[-1]).contiguous()


def _pad_to8(t: torch.Tensor, dim: int) -> torch.Tensor:
    """Zero-pad `dim` (a reduction dim) up to a multiple of 8: the tcgen05 GEMM takes K in
    16-byte steps, and zero rows / columns add nothing to the product."""
    k = t.shape[dim]
    if k % 8 == 0:
        return t
    pad = [0, 0] * (t.dim() - 1 - dim) + [0, 8 - k % 8]
    return torch.nn.functional.pad(t, pad).contiguous()


def mm_nt(a: torch.Tensor, b: torch.Tensor, residual: torch.Tensor | None = None, out_f32: bool = False,
          out: torch.Tensor | None = None) -> torch.Tensor:
    if not _ext.use_cuda(a):
        y = a @ b.t()
        if residual is not None:
            y = y + residual
        return y.float() if out_f32 else y
    C = _ext.load()
    a = _pad_to8(_c2d(a), 1)
    b = _pad_to8(b.contiguous(), 1)
    M, N = a.shape[0], b.shape[0]
    if out is None:
        out = torch.empty(M, N, device=a.device, dtype=torch.float32 if out_f32 else torch.bfloat16)
    if M <= FEW_ROW_LIBRARY_MAX and not out_f32 and a.dtype == b.dtype == torch.bfloat16:
        if residual is not None:
            return torch.addmm(_c2d(residual), a, b.t(), out=out)
        return torch.mm(a, b.t(), out=out)
    if residual is not None:
        C.gemm(a, b, out, False, False, EPI_ADD, 1.0, _c2d(residual), None, 256)
    else:
        C.gemm(a, b, out, False, False, EPI_F32 if out_f32 else EPI_BF16, 1.0, None, None, 256)
    return out


def mm_nn(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if not _ext.use_cuda(a):
        return a @ b
    C = _ext.load()
    a = _pad_to8(_c2d(a), 1)
    b = _pad_to8(b.contiguous(), 0)
    out = torch.empty(a.shape[0], b.shape[1], device=a.device, dtype=torch.bfloat16)
    C.gemm(a, b, out, False, True, EPI_BF16, 1.0, None, None, 256)
    return out


def mm_tn(a: torch.Tensor, b: torch.Tensor, out_f32: bool = False, accumulate_into: torch.Tensor | None = None
          ) -> torch.Tensor:
    if not _ext.use_cuda(a):
        y = a.t() @ b
        if accumulate_into is not None:
            accumulate_into += y
            return accumulate_into
        return y.float() if out_f32 else y
    C = _ext.load()
    a = _pad_to8(_c2d(a), 0)
    b = _pad_to8(_c2d(b), 0)
    if accumulate_into is not None:
        C.gemm(a, b, accumulate_into, True, True, EPI_ACC_F32, 1.0, None, None, 256)
        return accumulate_into
    out = torch.empty(a.shape[1], b.shape[1], device=a.device, dtype=torch.float32 if out_f32 else torch.bfloat16)
    C.gemm(a, b, out, True, True, EPI_F32 if out_f32 else EPI_BF16, 1.0, None, None, 256)
    return out


def interleave_gate_up(w1: torch.Tensor, w3: torch.Tensor, block: int = 32) -> torch.Tensor:
    """Stack gate (w1) and up (w3) rows interleaved in blocks of `block` rows:
    [w1[0:32], w3[0:32], w1[32:64], w3[32:64], ...].  Works on [F, D] or [E, F, D]."""
    F = w1.shape[-2]
    assert F % block == 0, "ffn dim must be a multiple of 32"
    lead = w1.shape[:-2]
    a = w1.reshape(*lead, F // block, 1, block, w1.shape[-1])
    b = w3.reshape(*lead, F // block, 1, block, w3.shape[-1])
    return torch.cat([a, b], dim=-3).reshape(*lead, 2 * F, w1.shape[-1])


def split_gate_up(w13: torch.Tensor, block: int = 32) -> tuple[torch.Tensor, torch.Tensor]:
    """Inverse of :func:`interleave_gate_up`."""
    F2 = w13.shape[-2]
    lead = w13.shape[:-2]
    v = w13.reshape(*lead, F2 // (2 * block), 2, block, w13.shape[-1])
    return (v[..., 0, :, :].reshape(*lead, F2 // 2, w13.shape[-1]),
            v[..., 1, :, :].reshape(*lead, F2 // 2, w13.shape[-1]))


def deinterleave_cols(h: torch.Tensor, block: int = 32) -> tuple[torch.Tensor, torch.Tensor]:
    """Split an activation laid out [g(32) u(32) g(32) u(32) ...] along the last dim."""
    F2 = h.shape[-1]
    v = h.reshape(*h.shape[:-1], F2 // (2 * block), 2, block)
    return v[..., 0, :].reshape(*h.shape[:-1], F2 // 2), v[..., 1, :].reshape(*h.shape[:-1], F2 // 2)


def interleave_cols(g: torch.Tensor, u: torch.Tensor, block: int = 32) -> torch.Tensor:
    F = g.shape[-1]
    a = g.reshape(*g.shape[:-1], F // block, 1, block)
    b = u.reshape(*u.shape[:-1], F // block, 1, block)
    return torch.cat([a, b], dim=-2).reshape(*g.shape[:-1], 2 * F)
