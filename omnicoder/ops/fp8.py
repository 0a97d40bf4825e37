"""Block-scaled fp8 (e4m3) linear algebra: 1 x 128 activation scales and
128 x 128 weight scales with fp32 scale factors, the tile scheme of block-scaled
fp8 training recipes.

  quantize_act(x [M, K])         -> (xq e4m3 [M, K], sx fp32 [K/128, M padded to 128])
  quantize_weight(w [(G,) N, K]) -> (wq e4m3, sw fp32 [G, ceil(N/128), K/128])
  fp8_mm(x, wq, sw)              -> x @ dequant(w)^T in bf16 (x quantised on the fly)
  fp8_grouped_mm(x_perm, wq, sw, offsets, rows) -> per-expert products (row groups of
                                    x_perm given by offsets, multiples of 128)

CUDA: the tcgen05 kind::f8f6f4 kernel of gemm_fp8.cu (per-K-block partial products
scaled and accumulated in fp32 by the epilogue warps).  CPU: dequantise and
matmul in fp32 (the oracle).  Scales are max|block| / 448 (e4m3's largest finite
value); an all-zero block gets scale 1.
"""
from __future__ import annotations

import torch

from . import _ext

E4M3 = torch.float8_e4m3fn
E4M3_MAX = 448.0


def _pad128(n: int) -> int:
    return (n + 127) // 128 * 128


def quantize_act_torch(x: torch.Tensor):
    M, K = x.shape
    xb = x.float().view(M, K // 128, 128)
    amax = xb.abs().amax(-1)
    scale = torch.where(amax > 0, amax * (1.0 / E4M3_MAX), torch.ones_like(amax))
    xq = (xb / scale[..., None]).to(E4M3).view(M, K)
    sx = torch.zeros(K // 128, _pad128(M), device=x.device)
    sx[:, :M] = scale.t()
    return xq, sx


def quantize_weight_torch(w: torch.Tensor):
    squeeze = w.dim() == 2
    w3 = w[None] if squeeze else w
    G, N, K = w3.shape
    Np = _pad128(N)
    wp = torch.zeros(G, Np, K, device=w.device, dtype=torch.float32)
    wp[:, :N] = w3.float()
    blocks = wp.view(G, Np // 128, 128, K // 128, 128)
    amax = blocks.abs().amax(dim=(2, 4))
    scale = torch.where(amax > 0, amax * (1.0 / E4M3_MAX), torch.ones_like(amax))
    q = (blocks / scale[:, :, None, :, None]).to(E4M3).view(G, Np, K)[:, :N]
    return (q[0] if squeeze else q).contiguous(), scale


def dequantize_act(xq: torch.Tensor, sx: torch.Tensor) -> torch.Tensor:
    M, K = xq.shape
    return (xq.float().view(M, K // 128, 128) * sx[:, :M].t()[..., None]).view(M, K)


def dequantize_weight(wq: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    squeeze = wq.dim() == 2
    w3 = wq[None] if squeeze else wq
    G, N, K = w3.shape
    s = sw.repeat_interleave(128, dim=1)[:, :N].repeat_interleave(128, dim=2)
    out = w3.float() * s
    return out[0] if squeeze else out


def quantize_act(x: torch.Tensor):
    if not _ext.use_cuda(x):
        return quantize_act_torch(x)
    return tuple(_ext.load().fp8_quant_act(x.contiguous()))


def quantize_weight(w: torch.Tensor):
    if not _ext.use_cuda(w):
        return quantize_weight_torch(w)
    wq, sw = _ext.load().fp8_quant_weight(w.contiguous())
    return wq, sw


def fp8_mm(x: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    """x [M, K] (bf16) @ dequant(wq, sw)^T -> [M, N] bf16, x quantised per 1 x 128 block."""
    xq, sx = quantize_act(x)
    if not _ext.use_cuda(x):
        return (dequantize_act(xq, sx) @ dequantize_weight(wq, sw).t()).to(x.dtype)
    out = torch.empty(x.shape[0], wq.shape[-2], device=x.device, dtype=torch.bfloat16)
    _ext.load().fp8_gemm(xq, sx, wq, sw.reshape(-1), out)
    return out


def fp8_grouped_mm(x_perm: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor, offsets: torch.Tensor,
                   rows: int) -> torch.Tensor:
    """Row group g of x_perm (rows [offsets[g], offsets[g+1]), multiples of 128) times
    dequant(wq[g])^T -> [rows, N] bf16."""
    xq, sx = quantize_act(x_perm)
    if not _ext.use_cuda(x_perm):
        w = dequantize_weight(wq, sw)
        xd = dequantize_act(xq, sx)
        out = torch.zeros(x_perm.shape[0], wq.shape[-2], dtype=torch.float32)
        off = offsets.tolist()
        for g in range(wq.shape[0]):
            out[off[g]:off[g + 1]] = xd[off[g]:off[g + 1]] @ w[g].t()
        return out.to(x_perm.dtype)
    out = torch.empty(x_perm.shape[0], wq.shape[-2], device=x_perm.device, dtype=torch.bfloat16)
    _ext.load().fp8_gemm(xq, sx, wq, sw.reshape(-1), out, offsets, rows)
    return out
