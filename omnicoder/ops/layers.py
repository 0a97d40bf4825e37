"""Autograd functions of the dense hot ops: linear (+ fused residual), RMSNorm
(+ fused residual add), LayerNorm, RoPE, embedding and the fused SwiGLU MLP.

Each function runs the sm_100a kernels when its input is on a CUDA device and a
plain PyTorch implementation on CPU.  The CPU implementation doubles as the
fp32 oracle of the kernel tests.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _ext
from .gemm import EPI_SWIGLU, EPI_SWIGLU_BWD, interleave_cols, deinterleave_cols, mm_nn, mm_nt, mm_tn


def _flat(t: torch.Tensor) -> torch.Tensor:
    return t.reshape(-1, t.shape[-1])


# ----------------------------------------------------------------------------
# Linear: y = x W^T (+ residual)
# ----------------------------------------------------------------------------
class _LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, residual):
        x2 = _flat(x).contiguous()
        y = mm_nt(x2, w, residual=None if residual is None else _flat(residual).contiguous())
        ctx.save_for_backward(x2, w)
        ctx.has_res = residual is not None
        return y.view(*x.shape[:-1], w.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w = ctx.saved_tensors
        dy2 = _flat(dy).contiguous()
        dx = mm_nn(dy2, w) if ctx.needs_input_grad[0] else None
        dw = mm_tn(dy2, x2) if ctx.needs_input_grad[1] else None
        dres = dy if ctx.has_res else None
        if dx is not None:
            dx = dx.view(*dy.shape[:-1], w.shape[1])
        return dx, dw, dres


def linear(x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
    """y = x @ w.T (+ residual), w [out, in]."""
    if not x.is_cuda:
        y = F.linear(x, w)
        return y if residual is None else y + residual
    return _LinearFn.apply(x, w, residual)


# ----------------------------------------------------------------------------
# RMSNorm (+ residual add)
# ----------------------------------------------------------------------------
class _RMSNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, residual, eps):
        C = _ext.load()
        xs = _flat(x).contiguous()
        if residual is not None:
            y, rstd, h = C.rmsnorm_fwd(xs, _flat(residual).contiguous(), w, eps)
        else:
            y, rstd = C.rmsnorm_fwd(xs, None, w, eps)
            h = xs
        ctx.save_for_backward(h, w, rstd)
        ctx.has_res = residual is not None
        ctx.shape = x.shape
        if residual is not None:
            return y.view(x.shape), h.view(x.shape)
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy, dh=None):
        h, w, rstd = ctx.saved_tensors
        C = _ext.load()
        dres = None if (not ctx.has_res or dh is None) else _flat(dh).contiguous()
        dx, dw = C.rmsnorm_bwd(h, w, rstd, _flat(dy).contiguous(), dres)
        dx = dx.view(ctx.shape)
        dwt = dw.to(w.dtype)
        if ctx.has_res:
            return dx, dwt, dx, None
        return dx, dwt, None, None


class _SplitNormFn(torch.autograd.Function):
    """(rms_norm(x[:, :n]) * w, x[:, n:]) of x [T, n + m] with one gradient for x."""

    @staticmethod
    def forward(ctx, x, w, n, eps):
        C = _ext.load()
        xa = x[:, :n].contiguous()
        y, rstd = C.rmsnorm_fwd(xa, None, w, eps)
        ctx.save_for_backward(xa, w, rstd)
        ctx.m = x.shape[1] - n
        return y, x[:, n:].contiguous()

    @staticmethod
    def backward(ctx, dy, dtail):
        xa, w, rstd = ctx.saved_tensors
        C = _ext.load()
        if dy is None:
            dy = torch.zeros_like(xa)
        dx, dw = C.rmsnorm_bwd(xa, w, rstd, dy.contiguous(), None)
        if dtail is None:
            dtail = torch.zeros(xa.shape[0], ctx.m, device=xa.device, dtype=xa.dtype)
        return torch.cat([dx, dtail], dim=1), dw.to(w.dtype), None, None


def split_norm(x: torch.Tensor, w: torch.Tensor, n: int, eps: float = 1e-6):
    """(RMSNorm of the first n columns of x, the remaining columns), both contiguous."""
    if not x.is_cuda:
        return rms_norm(x[:, :n], w, eps), x[:, n:]
    return _SplitNormFn.apply(x, w, n, eps)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float = 1e-6, residual: torch.Tensor | None = None):
    """RMSNorm(x (+ residual)) * w.  With `residual` returns (y, h) where h = x + residual."""
    if not x.is_cuda:
        h = x if residual is None else x + residual
        hf = h.float()
        y = (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + eps)).to(h.dtype) * w
        return y if residual is None else (y, h)
    return _RMSNormFn.apply(x, w, residual, eps)


class _LayerNormFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps):
        C = _ext.load()
        xs = _flat(x).contiguous()
        y, mean, rstd = C.layernorm_fwd(xs, w, b, eps)
        ctx.save_for_backward(xs, w, mean, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        xs, w, mean, rstd = ctx.saved_tensors
        dx, dw, db = _ext.load().layernorm_bwd(xs, w, mean, rstd, _flat(dy).contiguous())
        return dx.view(ctx.shape), dw.to(w.dtype), db.to(w.dtype), None


def layer_norm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float = 1e-5) -> torch.Tensor:
    if not x.is_cuda:
        return F.layer_norm(x, (x.shape[-1],), w, b, eps)
    return _LayerNormFn.apply(x, w, b, eps)


# ----------------------------------------------------------------------------
# RoPE
# ----------------------------------------------------------------------------
class RopeTable:
    """cos/sin table [2, max_pos, rot/2] (fp32) for rotary embeddings.

    inv_freq_i = theta^(-2i/rot); angle = (pos / scale) * inv_freq_i.  Same
    frequency formula as the reference (src/omnicoder/modeling/attention.py:115-160).
    """

    def __init__(self, rot: int, max_pos: int, theta: float = 10000.0, scale: float = 1.0, device=None):
        self.rot = rot
        self.max_pos = max_pos
        inv = theta ** (-torch.arange(0, rot, 2, dtype=torch.float64) / rot)
        t = torch.arange(max_pos, dtype=torch.float64) / scale
        ang = torch.outer(t, inv)
        self.cs = torch.stack([ang.cos(), ang.sin()]).float().contiguous()
        if device is not None:
            self.cs = self.cs.to(device)

    def to(self, device):
        if self.cs.device != torch.device(device):
            self.cs = self.cs.to(device)
        return self


def _rope_torch(x: torch.Tensor, cs: torch.Tensor, pos: torch.Tensor, interleaved: bool, sign: float) -> torch.Tensor:
    """x [..., T, rot] rotated by angle(pos[T]); returns a new tensor."""
    c = cs[0][pos].to(x.dtype)
    s = cs[1][pos].to(x.dtype) * sign
    if interleaved:
        x0, x1 = x[..., 0::2], x[..., 1::2]
        y0 = x0 * c - x1 * s
        y1 = x1 * c + x0 * s
        return torch.stack([y0, y1], dim=-1).flatten(-2)
    h = x.shape[-1] // 2
    x0, x1 = x[..., :h], x[..., h:]
    return torch.cat([x0 * c - x1 * s, x1 * c + x0 * s], dim=-1)


class _RopeFn(torch.autograd.Function):
    """Rotates x[..., off:off+rot] of every head in place (x is [T, H, hd] viewed)."""

    @staticmethod
    def forward(ctx, x, table, pos, pos0, seq, off, interleaved, heads):
        C = _ext.load()
        T, H, hd = x.shape
        H = heads if heads > 0 else H
        ctx.heads = H
        y = x
        C.rope(y, table.cs, pos, pos0, seq, T, H, y.stride(0), y.stride(1), off, table.rot, interleaved, 1.0)
        ctx.table, ctx.pos, ctx.pos0, ctx.seq, ctx.off, ctx.inter = table, pos, pos0, seq, off, interleaved
        ctx.mark_dirty(x)
        return y

    @staticmethod
    def backward(ctx, dy):
        C = _ext.load()
        d = dy.contiguous().clone()
        T = d.shape[0]
        C.rope(d, ctx.table.cs, ctx.pos, ctx.pos0, ctx.seq, T, ctx.heads, d.stride(0), d.stride(1), ctx.off,
               ctx.table.rot, ctx.inter, -1.0)
        return d, None, None, None, None, None, None, None


def apply_rope(x: torch.Tensor, table: RopeTable, positions: torch.Tensor | None = None, pos0: int = 0,
               seq: int = 0, off: int = 0, interleaved: bool = False, heads: int = 0) -> torch.Tensor:
    """Rotate dims [off, off+rot) of the first `heads` heads (0: all) of x [T, H, hd]
    (tokens flattened over the batch).  Position of token t: positions[t] if given,
    else pos0 + t % seq.  Returns x (rotated in place on CUDA, a new tensor on CPU)."""
    T = x.shape[0]
    nh = heads if heads > 0 else x.shape[1]
    if positions is None:
        s = seq if seq > 0 else T
        positions = (pos0 + torch.arange(T, device=x.device) % s)
    if not x.is_cuda:
        rot = table.rot
        xh = x[:, :nh]
        part = xh[..., off:off + rot]
        c = table.cs.to(x.device)
        rotated = _rope_torch(part.transpose(0, 1), c, positions.long(), interleaved, 1.0).transpose(0, 1)
        y = torch.cat([xh[..., :off], rotated, xh[..., off + rot:]], dim=-1)
        return y if nh == x.shape[1] else torch.cat([y, x[:, nh:]], dim=1)
    table.to(x.device)
    pos = positions.to(device=x.device, dtype=torch.int32).contiguous()
    return _RopeFn.apply(x, table, pos, 0, 1, off, interleaved, nh)


# ----------------------------------------------------------------------------
# Linear + RoPE: y = rope(x W^T) on `rope_heads` heads of `head_dim` at [off, off+rot)
# ----------------------------------------------------------------------------
class _LinearRopeFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, table, pos, head_dim, rope_heads, off, interleaved):
        C = _ext.load()
        x2 = _flat(x).contiguous()
        y = mm_nt(x2, w)
        T = y.shape[0]
        nh = y.shape[1] // head_dim
        C.rope(y, table.cs, pos, 0, 1, T, rope_heads, y.stride(0), head_dim, off, table.rot, interleaved, 1.0)
        ctx.save_for_backward(x2, w, pos)
        ctx.cfg = (table, head_dim, rope_heads, off, interleaved)
        ctx.xshape = x.shape
        return y

    @staticmethod
    def backward(ctx, dy):
        x2, w, pos = ctx.saved_tensors
        table, head_dim, rope_heads, off, interleaved = ctx.cfg
        C = _ext.load()
        d = dy.contiguous().clone()
        T = d.shape[0]
        C.rope(d, table.cs, pos, 0, 1, T, rope_heads, d.stride(0), head_dim, off, table.rot, interleaved, -1.0)
        dx = mm_nn(d, w).view(*ctx.xshape[:-1], w.shape[1]) if ctx.needs_input_grad[0] else None
        dw = mm_tn(d, x2) if ctx.needs_input_grad[1] else None
        return dx, dw, None, None, None, None, None, None


def linear_rope(x: torch.Tensor, w: torch.Tensor, table: RopeTable, positions: torch.Tensor, head_dim: int,
                rope_heads: int, off: int = 0, interleaved: bool = False) -> torch.Tensor:
    """y = x @ w.T viewed as [T, heads, head_dim]; dims [off, off+rot) of the first
    `rope_heads` heads are rotated by the position of each token.  Returns [T, heads*head_dim]."""
    if not x.is_cuda:
        y = F.linear(_flat(x), w)
        T = y.shape[0]
        nh = y.shape[1] // head_dim
        return apply_rope(y.view(T, nh, head_dim), table, positions, off=off, interleaved=interleaved,
                          heads=rope_heads).reshape(T, nh * head_dim)
    table.to(x.device)
    pos = positions.to(device=x.device, dtype=torch.int32).contiguous()
    return _LinearRopeFn.apply(x, w, table, pos, head_dim, rope_heads, off, interleaved)


# ----------------------------------------------------------------------------
# Embedding
# ----------------------------------------------------------------------------
class _EmbeddingFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, ids, w):
        ids_c = ids.contiguous().long()
        out = _ext.load().embedding_fwd(ids_c, w)
        ctx.save_for_backward(ids_c)
        ctx.wshape, ctx.wdtype = w.shape, w.dtype
        return out

    @staticmethod
    def backward(ctx, dout):
        (ids,) = ctx.saved_tensors
        dw = torch.zeros(ctx.wshape, device=dout.device, dtype=torch.float32)
        _ext.load().embedding_bwd(ids, dout.contiguous(), dw)
        return None, dw.to(ctx.wdtype)


def embedding(ids: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    if not w.is_cuda:
        return F.embedding(ids, w)
    return _EmbeddingFn.apply(ids, w)


# ----------------------------------------------------------------------------
# Fused SwiGLU MLP: y = (silu(x W1^T) * (x W3^T)) W2^T (+ residual)
# w13: gate/up rows interleaved in blocks of 32 ([2F, D]); w2: [D, F]
# ----------------------------------------------------------------------------
class _SwiGLUMLPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w13, w2, residual):
        C = _ext.load()
        x2 = _flat(x).contiguous()
        T = x2.shape[0]
        F2 = w13.shape[0]
        act = torch.empty(T, F2 // 2, device=x.device, dtype=torch.bfloat16)
        # the pre-activation is kept only for backward (without it, few-row calls take the
        # swap-AB kernel)
        H = torch.empty(T, F2, device=x.device, dtype=torch.bfloat16) if any(ctx.needs_input_grad) else None
        C.gemm(x2, w13, act, False, False, EPI_SWIGLU, 1.0, None, H, 256)
        y = mm_nt(act, w2, residual=None if residual is None else _flat(residual).contiguous())
        ctx.save_for_backward(x2, w13, w2, H, act)
        ctx.has_res = residual is not None
        return y.view(*x.shape[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, dy):
        x2, w13, w2, H, act = ctx.saved_tensors
        C = _ext.load()
        dy2 = _flat(dy).contiguous()
        T = dy2.shape[0]
        dw2 = mm_tn(dy2, act)
        dH = torch.empty(T, H.shape[1], device=dy.device, dtype=torch.bfloat16)
        C.gemm(dy2, w2, dH, False, True, EPI_SWIGLU_BWD, 1.0, H, None, 256)
        dx = mm_nn(dH, w13).view(*dy.shape[:-1], w13.shape[1])
        dw13 = mm_tn(dH, x2)
        return dx, dw13, dw2, (dy if ctx.has_res else None)


def swiglu_mlp(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, residual: torch.Tensor | None = None):
    if not x.is_cuda:
        h = F.linear(x, w13)
        g, u = deinterleave_cols(h)
        y = F.linear(F.silu(g) * u, w2)
        return y if residual is None else y + residual
    if not torch.is_grad_enabled():
        # inference: no pre-activation is kept, so few-row calls take the swap-AB kernel
        C = _ext.load()
        x2 = _flat(x).contiguous()
        act = torch.empty(x2.shape[0], w13.shape[0] // 2, device=x.device, dtype=torch.bfloat16)
        C.gemm(x2, w13, act, False, False, EPI_SWIGLU, 1.0, None, None, 256)
        y = mm_nt(act, w2, residual=None if residual is None else _flat(residual).contiguous())
        return y.view(*x.shape[:-1], w2.shape[0])
    return _SwiGLUMLPFn.apply(x, w13, w2, residual)


__all__ = ["linear", "linear_rope", "rms_norm", "layer_norm", "RopeTable", "apply_rope", "embedding", "swiglu_mlp",
           "interleave_cols", "deinterleave_cols"]
