"""Post-training weight quantisation for export (reference export AWQ / GPTQ
entry points, quant/int4_linear.py).

gptq_quantize(W, X, bits, group): the GPTQ algorithm (Frantar et al., 2022):
columns of W are quantised one at a time in the order of the inverse-Hessian
Cholesky factor of H = 2 X^T X (+ damping); each column's quantisation error
is propagated to the not-yet-quantised columns.  Symmetric per-row scales per
`group` input columns.  Returns (q int8 codes, scales [out, in/group]) and the
dequantised weight.
awq_scales(W, X, bits): activation-aware per-input-channel scaling
(Lin et al., 2023): s = mean|X|^alpha with alpha searched on a grid to
minimise || X W^T - Q(W * s) (X / s)^T ||; the returned weight is W * s and the
activations are divided by s (folded into the previous layer at export).
rtn_quantize: round-to-nearest baseline with the same format.
"""
from __future__ import annotations

import torch


def _qrange(bits: int) -> int:
    return 2 ** (bits - 1) - 1


def rtn_quantize(W: torch.Tensor, bits: int = 4, group: int = 128):
    out_f, in_f = W.shape
    qmax = _qrange(bits)
    Wg = W.float().view(out_f, in_f // group, group)
    scale = Wg.abs().amax(-1).clamp_min(1e-8) / qmax
    q = torch.round(Wg / scale[..., None]).clamp(-qmax, qmax)
    return q.view(out_f, in_f).to(torch.int8), scale, (q * scale[..., None]).view(out_f, in_f)


@torch.no_grad()
def gptq_quantize(W: torch.Tensor, X: torch.Tensor, bits: int = 4, group: int = 128, damp: float = 0.01,
                  block: int = 128):
    W = W.float().clone()
    out_f, in_f = W.shape
    qmax = _qrange(bits)
    H = 2.0 * X.float().t() @ X.float()
    dead = torch.diag(H) == 0
    H[dead, dead] = 1.0
    W[:, dead] = 0.0
    H += damp * torch.mean(torch.diag(H)) * torch.eye(in_f, device=W.device)
    Hinv = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(H)), upper=True)
    Q = torch.zeros_like(W)
    scales = torch.zeros(out_f, in_f // group, device=W.device)
    for i1 in range(0, in_f, block):
        i2 = min(i1 + block, in_f)
        W1 = W[:, i1:i2].clone()
        Q1 = torch.zeros_like(W1)
        Err1 = torch.zeros_like(W1)
        Hinv1 = Hinv[i1:i2, i1:i2]
        for i in range(i2 - i1):
            col = i1 + i
            if col % group == 0:       # scale of this group from the current (error-updated) weights
                g = W[:, col:col + group].clone()
                g[:, :i2 - col] = W1[:, i:i + min(group, i2 - col)] if col + group > i2 else W1[:, i:i + group]
                scales[:, col // group] = g.abs().amax(-1).clamp_min(1e-8) / qmax
            s = scales[:, col // group]
            w = W1[:, i]
            d = Hinv1[i, i]
            q = torch.round(w / s).clamp(-qmax, qmax) * s
            Q1[:, i] = q
            err = (w - q) / d
            W1[:, i:] -= err[:, None] * Hinv1[i, i:][None, :]
            Err1[:, i] = err
        Q[:, i1:i2] = Q1
        W[:, i2:] -= Err1 @ Hinv[i1:i2, i2:]
    codes = torch.round(Q.view(out_f, in_f // group, group) / scales[..., None]).clamp(-qmax, qmax)
    return codes.view(out_f, in_f).to(torch.int8), scales, Q


@torch.no_grad()
def awq_scales(W: torch.Tensor, X: torch.Tensor, bits: int = 4, group: int = 128, grid: int = 11):
    Wf, Xf = W.float(), X.float()
    ref = Xf @ Wf.t()
    mag = Xf.abs().mean(0).clamp_min(1e-6)
    best = (float("inf"), torch.ones_like(mag))
    for j in range(grid):
        alpha = j / (grid - 1)
        s = mag.pow(alpha)
        s = s / (s.max() * s.min()).sqrt()
        _, _, Wq = rtn_quantize(Wf * s[None, :], bits, group)
        err = (ref - (Xf / s[None, :]) @ Wq.t()).pow(2).mean().item()
        if err < best[0]:
            best = (err, s)
    return best[1], Wf * best[1][None, :]
