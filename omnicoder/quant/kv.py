"""Per-group KV quantisation (u8 min/max, nf4 codebook) and a paged latent KV
store -- the reference's KV-cache formats (src/omnicoder/modeling/quant/
kv_cache.py:46-257), used for export sidecars and ONNX-runtime style paging.

The batched decode path of this framework keeps its cache in int8 with one
symmetric scale per token (and head) instead (omnicoder.inference.kv_cache),
which the decode attention kernel dequantises in its inner loop.

Formats (last dim split in groups of `group_size`, padded with zeros):
  u8   scale = (max - min) / 255, zero = round(-min / scale) in [0, 255],
       q = clamp(round(x / scale + zero), 0, 255), x = (q - zero) * scale.
  nf4  mean and std per group, q = index of the nearest codebook entry to
       (x - mean) / std, x = code[q] * std + mean.  The 16-entry codebook is the
       reference's (kept identical so caches written by either side decode the
       same).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

NF4_CODEBOOK = torch.tensor([-1.078125, -0.8515625, -0.671875, -0.5234375, -0.39453125, -0.27734375, -0.1640625,
                             -0.0546875, 0.0546875, 0.1640625, 0.27734375, 0.39453125, 0.5234375, 0.671875,
                             0.8515625, 1.078125], dtype=torch.float32)


@dataclass
class KvQuantMeta:
    scheme: str
    group_size: int
    k_scale: torch.Tensor | None = None
    k_offset: torch.Tensor | None = None      # zero point (u8) or mean (nf4), [B, H, T, G]
    v_scale: torch.Tensor | None = None
    v_offset: torch.Tensor | None = None

    def to(self, device):
        for n in ("k_scale", "k_offset", "v_scale", "v_offset"):
            t = getattr(self, n)
            if t is not None:
                setattr(self, n, t.to(device))
        return self


def _groups(x: torch.Tensor, g: int):
    D = x.shape[-1]
    G = (D + g - 1) // g
    pad = G * g - D
    if pad:
        x = F.pad(x, (0, pad))
    return x.reshape(*x.shape[:-1], G, g), D


def _quant_one(x: torch.Tensor, scheme: str, g: int):
    xg, D = _groups(x.float(), g)
    if scheme == "u8":
        lo, hi = xg.amin(-1), xg.amax(-1)
        scale = (hi - lo).clamp_min(1e-8) / 255.0
        zero = (-lo / scale).round().clamp(0, 255)
        q = (xg / scale[..., None] + zero[..., None]).round().clamp(0, 255).to(torch.uint8)
        return q.reshape(*x.shape[:-1], -1)[..., :D], scale, zero
    if scheme == "nf4":
        mean = xg.mean(-1)
        std = ((xg - mean[..., None]) ** 2).mean(-1).clamp_min(1e-8).sqrt()
        z = (xg - mean[..., None]) / std[..., None]
        code = NF4_CODEBOOK.to(x.device)
        q = (z[..., None] - code).abs().argmin(-1).to(torch.uint8)
        return q.reshape(*x.shape[:-1], -1)[..., :D], std, mean
    raise ValueError(f"unknown KV quantisation scheme {scheme!r}")


def _dequant_one(q: torch.Tensor, scale: torch.Tensor, off: torch.Tensor, scheme: str, g: int, dtype):
    qg, D = _groups(q.float() if scheme == "u8" else q.long().float(), g)
    if scheme == "u8":
        x = (qg - off[..., None]) * scale[..., None]
    else:
        x = NF4_CODEBOOK.to(q.device)[qg.long()] * scale[..., None] + off[..., None]
    return x.reshape(*q.shape[:-1], -1)[..., :D].to(dtype)


@torch.no_grad()
def quantize_kv(k_lat: torch.Tensor, v_lat: torch.Tensor, scheme: str = "u8", group_size: int = 64):
    """k_lat, v_lat [B, H, T, D] -> (kq, vq (uint8), KvQuantMeta)."""
    kq, ks, ko = _quant_one(k_lat, scheme, group_size)
    vq, vs, vo = _quant_one(v_lat, scheme, group_size)
    return kq, vq, KvQuantMeta(scheme, group_size, ks, ko, vs, vo)


@torch.no_grad()
def dequantize_kv(kq: torch.Tensor, vq: torch.Tensor, meta: KvQuantMeta, dtype=torch.float32):
    return (_dequant_one(kq, meta.k_scale, meta.k_offset, meta.scheme, meta.group_size, dtype),
            _dequant_one(vq, meta.v_scale, meta.v_offset, meta.scheme, meta.group_size, dtype))


class PagedKvCache:
    """Latent K/V [B, H, T, D] kept in pages of `page_len` tokens (host memory),
    oldest pages evicted beyond `max_pages`; `materialize_tail(window)` returns the
    last `window` tokens."""

    def __init__(self, page_len: int = 256, max_pages: int = 128, device="cpu"):
        self.page_len, self.max_pages, self.device = page_len, max_pages, torch.device(device)
        self.pages: list[tuple[torch.Tensor, torch.Tensor]] = []

    def append_tokens(self, k_lat: torch.Tensor, v_lat: torch.Tensor) -> None:
        assert k_lat.shape == v_lat.shape
        T = k_lat.shape[2]
        o = 0
        while o < T:
            if self.pages and self.pages[-1][0].shape[2] < self.page_len:
                pk, pv = self.pages.pop()
                take = min(self.page_len - pk.shape[2], T - o)
                pk = torch.cat([pk, k_lat[:, :, o:o + take].to(self.device)], 2)
                pv = torch.cat([pv, v_lat[:, :, o:o + take].to(self.device)], 2)
            else:
                take = min(self.page_len, T - o)
                pk = k_lat[:, :, o:o + take].to(self.device)
                pv = v_lat[:, :, o:o + take].to(self.device)
            self.pages.append((pk, pv))
            if len(self.pages) > self.max_pages:
                self.pages.pop(0)
            o += take

    def __len__(self) -> int:
        return sum(p[0].shape[2] for p in self.pages)

    def materialize_tail(self, window: int):
        if not self.pages:
            raise ValueError("PagedKvCache is empty")
        ks, vs, total = [], [], 0
        for k, v in reversed(self.pages):
            need = window - total
            if need <= 0:
                break
            ks.append(k[:, :, -need:])
            vs.append(v[:, :, -need:])
            total += ks[-1].shape[2]
        return torch.cat(ks[::-1], 2), torch.cat(vs[::-1], 2)
