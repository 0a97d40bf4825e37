"""Gaussian splatting renderers (reference src/omnicoder/modeling/gaussian/renderer.py:12-235).

3D: camera transform X_c = X R^T + t, pinhole projection (u, v) = K [x/z, y/z, 1],
per-Gaussian pixel footprint scales s = sqrt(diag(Sigma)) * f / z; 2D: the means
are pixels and s = sqrt(diag(Sigma)).  Each Gaussian is splatted over a k x k
footprint (taps spaced by s), tap weight exp(-0.5 |offset / s|^2) * opacity;
colour, alpha and depth accumulate per pixel and are normalised by alpha.

CUDA + no gradient: the projection runs in torch, the splat in the sm_100a
kernel of gsplat.cu (fire-and-forget float reductions).  With gradients (or
on CPU) the same formulation runs with torch index_add so autograd reaches
positions, covariances, colours and opacities.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ..ops import _ext


def project_gaussians(pos, cov, cov_diag, rgb, K, R, t):
    """pos [B, N, 3] -> (u, v, z, sxx, syy) each [B, N]."""
    Xc = pos @ R.transpose(1, 2) + t[:, None, :]
    z = Xc[..., 2]
    zs = z.clamp_min(1e-6)
    xy1 = torch.stack([Xc[..., 0] / zs, Xc[..., 1] / zs, torch.ones_like(zs)], -1)
    uv = xy1 @ K.transpose(1, 2)
    if cov is not None:
        sxx, syy = cov[..., 0, 0], cov[..., 1, 1]
    else:
        cd = cov_diag if cov_diag is not None else rgb      # the reference falls back to the colours here
        sxx, syy = cd[..., 0], cd[..., 1]
    fx, fy = K[:, 0, 0][:, None], K[:, 1, 1][:, None]
    sx = sxx.clamp_min(1e-9).sqrt() * fx / zs
    sy = syy.clamp_min(1e-9).sqrt() * fy / zs
    return uv[..., 0], uv[..., 1], z, sx, sy


def splat_torch(u, v, sx, sy, opa, rgb, z, H: int, W: int, k: int):
    B, N = u.shape
    half = k // 2
    off = torch.arange(k, device=u.device) - half
    oy, ox = torch.meshgrid(off, off, indexing="ij")
    ox, oy = ox.reshape(1, 1, -1).to(u.dtype), oy.reshape(1, 1, -1).to(u.dtype)
    px = torch.round(u[..., None] + ox * sx[..., None]).long()
    py = torch.round(v[..., None] + oy * sy[..., None]).long()
    inside = (px >= 0) & (px < W) & (py >= 0) & (py < H)
    gx = ox / sx[..., None].clamp_min(1e-6)
    gy = oy / sy[..., None].clamp_min(1e-6)
    alpha = opa.reshape(B, N, 1) * torch.exp(-0.5 * (gx * gx + gy * gy)) * inside.to(u.dtype)
    lin = (py.clamp(0, H - 1) * W + px.clamp(0, W - 1)) + (torch.arange(B, device=u.device) * H * W).view(B, 1, 1)
    lin = lin.reshape(-1)
    a = alpha.reshape(-1)
    col = rgb.reshape(B, N, 1, 3).expand(B, N, k * k, 3).reshape(-1, 3)
    num = torch.zeros(B * H * W, 3, dtype=u.dtype, device=u.device).index_add(0, lin, a[:, None] * col)
    den = torch.zeros(B * H * W, dtype=u.dtype, device=u.device).index_add(0, lin, a)
    out = (num / den.clamp_min(1e-6)[:, None]).view(B, H, W, 3).permute(0, 3, 1, 2)
    if z is None:
        return out, None
    dn = torch.zeros(B * H * W, dtype=u.dtype, device=u.device).index_add(
        0, lin, (z[..., None].expand(B, N, k * k).reshape(-1)) * a)
    return out, (dn / den.clamp_min(1e-6)).view(B, 1, H, W)


def splat(u, v, sx, sy, opa, rgb, z, H, W, k):
    need_grad = torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (u, v, sx, sy, opa, rgb, z))
    if u.is_cuda and not need_grad:
        C = _ext.load()
        f = lambda t: t.float().contiguous()
        outs = C.gsplat_forward(f(u), f(v), f(sx), f(sy), f(opa.reshape(u.shape)), f(rgb), None if z is None else f(z),
                                H, W, k)
        return outs[0], (outs[1] if z is not None else None)
    return splat_torch(u, v, sx, sy, opa.reshape(u.shape), rgb, z, H, W, k)


class GaussianSplatRenderer3D(nn.Module):
    def __init__(self, kernel: int = 11):
        super().__init__()
        self.kernel = kernel if kernel % 2 == 1 else kernel + 1

    def forward(self, pos, cov, cov_diag, rgb, opa, K, R, t, image_size):
        u, v, z, sx, sy = project_gaussians(pos, cov, cov_diag, rgb, K, R, t)
        H, W = image_size
        return splat(u, v, sx, sy, opa, rgb, z, H, W, self.kernel)


class GaussianSplatRenderer2D(nn.Module):
    def __init__(self, kernel: int = 11):
        super().__init__()
        self.kernel = kernel if kernel % 2 == 1 else kernel + 1

    def forward(self, mean, cov_diag, rgb, opa, image_size):
        H, W = image_size
        sx = cov_diag[..., 0].clamp_min(1e-9).sqrt()
        sy = cov_diag[..., 1].clamp_min(1e-9).sqrt()
        return splat(mean[..., 0], mean[..., 1], sx, sy, opa, rgb, None, H, W, self.kernel)[0]
