"""Routed-expert FFN (top-k softmax router, SwiGLU experts) on one device.

CUDA path (all sm_100a kernels):
  router logits (tcgen05 GEMM, fp32 out) -> softmax/top-k/renorm -> deterministic
  permutation plan (128-row padded expert segments) -> gather -> grouped GEMM
  with fused SwiGLU (saves the pre-activation) -> grouped GEMM -> weighted
  combine (+ shared-expert/residual add).
Backward: combine^T (also the routing-weight gradient) -> grouped GEMM with the
fused SwiGLU backward -> grouped weight-gradient GEMMs -> un-permute ->
router backward (softmax, renorm, load-balance and z-loss terms) -> router GEMMs.

The reference's dispatch (src/omnicoder/modeling/kernels/moe_scatter.py:315-912)
keeps at most `top_k` tokens per expert and passes no gradient to experts or
routers (detached banks, moe_scatter.py:344-345; moe_layer.py:1056-1059); this
layer is dropless by default (or uses a capacity factor) and trains both.

CPU path: a readable per-expert loop, the fp32 oracle of the kernels.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _ext
from .gemm import EPI_BF16, EPI_SWIGLU, EPI_SWIGLU_BWD, deinterleave_cols, mm_nn, mm_nt, mm_tn


def cap_rows_for(tokens: int, k: int, n_experts: int, capacity: int) -> int:
    """Rows of the padded permuted buffer: every expert segment is rounded up to 128."""
    kept = tokens * k if capacity <= 0 else min(tokens * k, n_experts * capacity)
    return kept + n_experts * 128


def route_torch(logits: torch.Tensor, k: int, renorm: bool):
    """softmax over experts, top-k (ties -> lower expert id), optional renormalisation."""
    probs = torch.softmax(logits.float(), dim=-1)
    # stable tie-break toward the lower expert id
    w, idx = torch.topk(probs, k, dim=-1, sorted=True)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return idx, w, probs


def keep_mask_torch(idx: torch.Tensor, n_experts: int, capacity: int) -> torch.Tensor:
    """Pairs (t, k) in token order; the first `capacity` pairs of each expert are kept."""
    flat = idx.reshape(-1)
    if capacity <= 0:
        return torch.ones_like(flat, dtype=torch.bool).view_as(idx)
    onehot = F.one_hot(flat.long(), n_experts)
    rank = (onehot.cumsum(0) - 1).gather(1, flat.long().unsqueeze(1)).squeeze(1)
    return (rank < capacity).view_as(idx)


def moe_ffn_torch(x, router_w, w13, w2, k, capacity, renorm, aux_alpha=0.0, z_beta=0.0, add=None):
    """Reference MoE forward on any device with plain torch ops; returns (out, aux_loss)."""
    T, D = x.shape
    E = router_w.shape[0]
    logits = x.float() @ router_w.float().t()
    idx, w, probs = route_torch(logits, k, renorm)
    keep = keep_mask_torch(idx, E, capacity)
    out = torch.zeros(T, D, dtype=torch.float32, device=x.device)
    for e in range(E):
        sel = (idx == e) & keep
        tok, slot = sel.nonzero(as_tuple=True)
        if tok.numel() == 0:
            continue
        h = x[tok].float() @ w13[e].float().t()
        g, u = deinterleave_cols(h)
        y = (F.silu(g) * u) @ w2[e].float().t()
        out.index_add_(0, tok, y * w[tok, slot].unsqueeze(1))
    if add is not None:
        out = out + add.float()
    aux = x.new_zeros((), dtype=torch.float32)
    if aux_alpha > 0:
        counts = torch.bincount(idx.reshape(-1), minlength=E).float()
        f = (counts / (T * k)).detach()
        aux = aux + aux_alpha * E * (f * probs.mean(0)).sum()
    if z_beta > 0:
        lse = torch.logsumexp(logits, dim=-1)
        aux = aux + z_beta * (lse * lse).mean()
    return out.to(x.dtype), aux


_STATIC = {"on": False}


class static_shapes:
    """Context in which the routed experts run the static-shape formulation below (for graph
    exporters: torch.export, ONNX), i.e. without the capacity mask's data-dependent shapes."""

    def __enter__(self):
        self.prev = _STATIC["on"]
        _STATIC["on"] = True
        return self

    def __exit__(self, *exc):
        _STATIC["on"] = self.prev
        return False


def moe_ffn_static(x, router_w, w13, w2, k, renorm, add=None):
    """Dropless routed SwiGLU with shapes independent of the routing: every token's k expert
    weight matrices are gathered ([T, k, 2F, D], [T, k, D, F]) and applied with batched matmuls.
    Equal to moe_ffn_torch with capacity 0; meant for exported few-token decode steps."""
    T, D = x.shape
    logits = x.float() @ router_w.float().t()
    idx, w, _ = route_torch(logits, k, renorm)
    xe = x.float()[:, None, :, None].expand(T, k, D, 1)                       # [T, k, D, 1]
    h = torch.matmul(w13[idx].float(), xe).squeeze(-1)                         # [T, k, 2F]
    g, u = deinterleave_cols(h.reshape(T * k, -1))
    a = (F.silu(g) * u).reshape(T, k, -1, 1)                                   # [T, k, F, 1]
    y = torch.matmul(w2[idx].float(), a).squeeze(-1)                           # [T, k, D]
    out = (y * w[..., None]).sum(1)
    if add is not None:
        out = out + add.float()
    return out.to(x.dtype), x.new_zeros((), dtype=torch.float32)


class _MoEFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, router_w, w13, w2, add, k, capacity, renorm, aux_alpha, z_beta, grad_scale_aux):
        C = _ext.load()
        x = x.contiguous()
        T, D = x.shape
        E = router_w.shape[0]
        F2 = w13.shape[1]
        logits = mm_nt(x, router_w, out_f32=True)
        idx, wts, probs = C.router_topk(logits, k, renorm)
        rows = cap_rows_for(T, k, E, capacity)
        counts, offsets, pos, src = C.moe_plan(idx, E, capacity, rows)
        x_perm = torch.empty(rows, D, device=x.device, dtype=torch.bfloat16)
        C.moe_gather(x, src, x_perm, k, offsets)
        act = torch.empty(rows, F2 // 2, device=x.device, dtype=torch.bfloat16)
        H = torch.empty(rows, F2, device=x.device, dtype=torch.bfloat16)
        C.gemm_grouped_m(x_perm, w13, offsets, act, False, EPI_SWIGLU, 1.0, None, H, 256, rows)
        y_perm = torch.empty(rows, D, device=x.device, dtype=torch.bfloat16)
        C.gemm_grouped_m(act, w2, offsets, y_perm, False, EPI_BF16, 1.0, None, None, 256, rows)
        out = C.moe_combine(y_perm, pos, wts, None if add is None else add.contiguous())
        ctx.save_for_backward(x, router_w, w13, w2, logits, probs, idx, wts, counts, offsets, pos, src, x_perm, H,
                              act, y_perm)
        ctx.cfg = (k, capacity, renorm, aux_alpha, z_beta, grad_scale_aux, add is not None, rows)
        # logged value of the auxiliary losses (gradient is injected in backward)
        aux = x.new_zeros((), dtype=torch.float32)
        if aux_alpha > 0:
            f = counts.float() / (T * k)
            aux = aux + aux_alpha * E * (f * probs.mean(0)).sum()
        if z_beta > 0:
            lse = torch.logsumexp(logits, dim=-1)
            aux = aux + z_beta * (lse * lse).mean()
        ctx.mark_non_differentiable(aux)
        return out, aux

    @staticmethod
    def backward(ctx, dout, daux):
        (x, router_w, w13, w2, logits, probs, idx, wts, counts, offsets, pos, src, x_perm, H, act,
         y_perm) = ctx.saved_tensors
        k, capacity, renorm, aux_alpha, z_beta, gs, has_add, rows = ctx.cfg
        C = _ext.load()
        E = router_w.shape[0]
        dout = dout.contiguous()
        dy_perm, dwts = C.moe_combine_bwd(dout, y_perm, src, wts, offsets, k)
        dH = torch.empty_like(H)
        C.gemm_grouped_m(dy_perm, w2, offsets, dH, True, EPI_SWIGLU_BWD, 1.0, H, None, 256, rows)
        dw2 = torch.empty_like(w2)
        C.gemm_grouped_k(dy_perm, act, offsets, dw2, EPI_BF16, 1.0, 256)
        dx_perm = torch.empty_like(x_perm)
        C.gemm_grouped_m(dH, w13, offsets, dx_perm, True, EPI_BF16, 1.0, None, None, 256, rows)
        dw13 = torch.empty_like(w13)
        C.gemm_grouped_k(dH, x_perm, offsets, dw13, EPI_BF16, 1.0, 256)
        dlogits, _ = C.router_bwd(logits, probs, idx, dwts, counts, renorm, aux_alpha * gs, z_beta * gs)
        dx_router = mm_nn(dlogits, router_w)
        dx = C.moe_scatter_add(dx_perm, pos, dx_router)
        drouter = mm_tn(dlogits, x)
        return dx, drouter, dw13, dw2, (dout if has_add else None), None, None, None, None, None, None


SKINNY_MAX_PAIRS = 256   # token-expert pairs up to which inference uses the few-row expert GEMM


def _moe_infer(x, router_w, w13, w2, add, k, capacity, renorm):
    """Forward only (no autograd state).  Up to SKINNY_MAX_PAIRS routed pairs the
    permutation is packed (no 128-row padding) and both expert GEMMs run the
    few-row swap-AB kernel, which streams each expert's weights once whatever
    its token count; larger batches use the tile GEMM without storing the
    SwiGLU pre-activation."""
    C = _ext.load()
    x = x.contiguous()
    T, D = x.shape
    E = router_w.shape[0]
    F2 = w13.shape[1]
    logits = mm_nt(x, router_w, out_f32=True)
    idx, wts, _ = C.router_topk(logits, k, renorm)
    n = T * k
    dev = x.device
    if n <= SKINNY_MAX_PAIRS:
        counts, offsets, pos, src = C.moe_plan(idx, E, capacity, n, 1)
        x_perm = torch.empty(n, D, device=dev, dtype=torch.bfloat16)
        C.moe_gather(x, src, x_perm, k, offsets)
        act = torch.empty(n, F2 // 2, device=dev, dtype=torch.bfloat16)
        C.gemm_skinny_grouped(x_perm, w13, offsets, act, EPI_SWIGLU, 1.0, n)
        y_perm = torch.empty(n, D, device=dev, dtype=torch.bfloat16)
        C.gemm_skinny_grouped(act, w2, offsets, y_perm, EPI_BF16, 1.0, n)
    else:
        rows = cap_rows_for(T, k, E, capacity)
        counts, offsets, pos, src = C.moe_plan(idx, E, capacity, rows)
        x_perm = torch.empty(rows, D, device=dev, dtype=torch.bfloat16)
        C.moe_gather(x, src, x_perm, k, offsets)
        act = torch.empty(rows, F2 // 2, device=dev, dtype=torch.bfloat16)
        C.gemm_grouped_m(x_perm, w13, offsets, act, False, EPI_SWIGLU, 1.0, None, None, 256, rows)
        y_perm = torch.empty(rows, D, device=dev, dtype=torch.bfloat16)
        C.gemm_grouped_m(act, w2, offsets, y_perm, False, EPI_BF16, 1.0, None, None, 256, rows)
    out = C.moe_combine(y_perm, pos, wts, None if add is None else add.contiguous())
    return out, x.new_zeros((), dtype=torch.float32)


def moe_ffn(x: torch.Tensor, router_w: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, k: int,
            capacity: int = 0, renorm: bool = True, aux_alpha: float = 0.0, z_beta: float = 0.0,
            add: torch.Tensor | None = None, aux_grad_scale: float = 1.0):
    """Routed SwiGLU experts.  x [T, D]; router_w [E, D]; w13 [E, 2F, D] (gate/up rows
    interleaved by 32); w2 [E, D, F].  Returns (out [T, D] (+ add), aux_loss scalar).

    On CUDA the auxiliary-loss gradient (scaled by `aux_grad_scale`) is injected
    inside backward and the returned aux value is for logging; on CPU it is a
    differentiable scalar the caller adds to the loss."""
    if _STATIC["on"]:
        return moe_ffn_static(x, router_w, w13, w2, k, renorm, add)
    if not x.is_cuda:
        return moe_ffn_torch(x, router_w, w13, w2, k, capacity, renorm, aux_alpha, z_beta, add)
    if not (torch.is_grad_enabled() and any(t.requires_grad for t in (x, router_w, w13, w2))):
        return _moe_infer(x, router_w, w13, w2, add, k, capacity, renorm)
    return _MoEFn.apply(x, router_w, w13, w2, add, k, capacity, renorm, aux_alpha, z_beta, aux_grad_scale)
