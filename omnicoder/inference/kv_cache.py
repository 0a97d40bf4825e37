"""Key/value cache of the spec model family for batched generation.

Per layer:
  * MHA / GQA: keys and values [B, L, Hk, D] (bf16) or int8 with one fp32
    scale per (sequence, position, head).
  * MLA: the compressed latent [B, L, r + dr] = (normalised kv latent c,
    rotated rope key) shared by all heads (bf16) or int8 with one fp32 scale
    per (sequence, position).  Decoding attends over this latent directly
    (absorbed up-projections, see OmniLM.prepare_inference).

`lengths[b]` counts the cached positions of sequence b; writes go to
positions lengths[b] .. lengths[b]+T_new-1, stored at cache rows
`sink + position`.  With `cfg.attn.mem_slots` = M > 0 the first M rows hold
compressed memory: `compress_memory()` summarises the tokens that fell out of
the attention window into M segment means (the reference's CompressiveKV
segment pooling, src/omnicoder/modeling/memory.py:77-178, without its learned
gates), which every later query attends to.  Quantisation is symmetric:
q = round(x / s), s = max|x| / 127 over the quantised group (the reference
quantises per group of 64 with min/max zero points, src/omnicoder/modeling/
quant/kv_cache.py:108-257; the per-head per-token symmetric scale keeps the
dequantisation a single multiply inside the attention kernel).
"""
from __future__ import annotations

import torch

from ..config import ModelConfig


def quantize_int8(x: torch.Tensor, dim: int = -1) -> tuple[torch.Tensor, torch.Tensor]:
    """Symmetric int8 with one scale per slice along `dim` (reduced)."""
    amax = x.float().abs().amax(dim=dim, keepdim=True).clamp_min(1e-8)
    s = amax / 127.0
    q = torch.round(x.float() / s).clamp_(-127, 127).to(torch.int8)
    return q, s.squeeze(dim)


def dequantize_int8(q: torch.Tensor, s: torch.Tensor, dim: int = -1, dtype=torch.float32) -> torch.Tensor:
    return (q.float() * s.unsqueeze(dim)).to(dtype)


class KVCache:
    def __init__(self, cfg: ModelConfig, batch: int, max_len: int, device, dtype=None, kv_dtype: str = "bf16"):
        if dtype is None:
            dtype = torch.bfloat16 if str(device).startswith("cuda") else torch.float32
        self.cfg, self.batch, self.max_len, self.device, self.dtype = cfg, batch, max_len, torch.device(device), dtype
        assert kv_dtype in ("bf16", "int8"), kv_dtype
        self.kv_dtype = kv_dtype
        self.mla = cfg.attn.kind == "mla"
        self.sink = int(cfg.attn.mem_slots)          # rows reserved for compressed memory
        self.n_mem = 0                                # rows of memory currently valid
        self.lengths = torch.zeros(batch, dtype=torch.int32, device=device)
        self.k, self.v, self.ks, self.vs = [], [], [], []
        store = torch.int8 if kv_dtype == "int8" else dtype
        max_len = max_len + self.sink
        for _ in range(cfg.n_layers):
            if self.mla:
                w = cfg.attn.kv_lora_rank + cfg.attn.qk_rope_dim
                self.k.append(torch.zeros(batch, max_len, w, dtype=store, device=device))
                self.v.append(None)
                self.ks.append(torch.zeros(batch, max_len, dtype=torch.float32, device=device) if kv_dtype == "int8" else None)
                self.vs.append(None)
            else:
                Hk, D = cfg.n_kv_heads, cfg.head_dim
                self.k.append(torch.zeros(batch, max_len, Hk, D, dtype=store, device=device))
                self.v.append(torch.zeros(batch, max_len, Hk, D, dtype=store, device=device))
                if kv_dtype == "int8":
                    self.ks.append(torch.zeros(batch, max_len, Hk, dtype=torch.float32, device=device))
                    self.vs.append(torch.zeros(batch, max_len, Hk, dtype=torch.float32, device=device))
                else:
                    self.ks.append(None)
                    self.vs.append(None)

    # ------------------------------------------------------------------
    def positions(self, t_new: int) -> torch.Tensor:
        """[B, t_new] absolute positions of the next t_new tokens."""
        return self.lengths.long()[:, None] + torch.arange(t_new, device=self.device)[None, :]

    def write(self, layer: int, pos: torch.Tensor, k: torch.Tensor, v: torch.Tensor | None = None):
        """Store new entries at positions pos [B, T]; k [B, T, ...] (MLA: latent [B, T, r+dr])."""
        B, T = pos.shape
        if k.is_cuda and self.k[layer].dtype in (torch.int8, torch.bfloat16):
            from ..ops import _ext
            C = _ext.load()
            p = pos.to(torch.int64).contiguous()
            if self.mla:
                C.kv_cache_write(k.reshape(B, T, 1, -1).to(torch.bfloat16).contiguous(), p, self.k[layer],
                                 self.ks[layer], self.sink)
            else:
                C.kv_cache_write(k.to(torch.bfloat16).contiguous(), p, self.k[layer], self.ks[layer], self.sink)
                if v is not None:
                    C.kv_cache_write(v.to(torch.bfloat16).contiguous(), p, self.v[layer], self.vs[layer], self.sink)
            return
        pos = pos + self.sink
        bidx = torch.arange(B, device=self.device)[:, None].expand(B, T)
        if self.kv_dtype == "int8":
            if self.mla:
                q, s = quantize_int8(k, -1)
                self.k[layer][bidx, pos] = q
                self.ks[layer][bidx, pos] = s
            else:
                q, s = quantize_int8(k, -1)
                self.k[layer][bidx, pos] = q
                self.ks[layer][bidx, pos] = s
                q, s = quantize_int8(v, -1)
                self.v[layer][bidx, pos] = q
                self.vs[layer][bidx, pos] = s
        else:
            self.k[layer][bidx, pos] = k.to(self.k[layer].dtype)
            if v is not None:
                self.v[layer][bidx, pos] = v.to(self.v[layer].dtype)

    @torch.no_grad()
    def compress_memory(self, window: int) -> int:
        """Fill the memory rows with segment means of the tokens older than the window
        (positions [0, min(lengths) - window)); returns the number of valid memory rows."""
        M = self.sink
        n_old = int(self.lengths.min()) - window
        if M == 0 or n_old <= 0:
            self.n_mem = 0
            return 0
        bounds = [(i * n_old) // M for i in range(M + 1)]
        for layer in range(self.cfg.n_layers):
            for store, scale in ((self.k, self.ks), (self.v, self.vs)):
                t = store[layer]
                if t is None:
                    continue
                rows = t[:, M:M + n_old].float()
                if scale[layer] is not None:
                    rows = rows * scale[layer][:, M:M + n_old].unsqueeze(-1)
                segs = torch.stack([rows[:, a:max(b, a + 1)].mean(1) for a, b in zip(bounds[:-1], bounds[1:])], 1)
                if scale[layer] is not None:
                    q, sc = quantize_int8(segs, -1)
                    t[:, :M] = q
                    scale[layer][:, :M] = sc
                else:
                    t[:, :M] = segs.to(t.dtype)
        self.n_mem = M
        return M

    def advance(self, t_new: int):
        self.lengths += t_new

    def rollback(self, new_lengths: torch.Tensor):
        """Forget positions >= new_lengths[b] (speculative decoding rejection)."""
        self.lengths.copy_(new_lengths.to(self.lengths.dtype))

    def reorder(self, index: torch.Tensor):
        """Keep / permute sequences (beam search or finished-sequence compaction)."""
        for lst in (self.k, self.v, self.ks, self.vs):
            for i, t in enumerate(lst):
                if t is not None:
                    lst[i] = t.index_select(0, index)
        self.lengths = self.lengths.index_select(0, index)
        self.batch = int(index.numel())

    def view(self, b0: int, b1: int) -> "KVCache":
        """A cache over sequences [b0, b1) that shares this cache's storage (for chunked prefill)."""
        v = object.__new__(KVCache)
        v.__dict__.update(self.__dict__)
        v.batch = b1 - b0
        v.lengths = self.lengths[b0:b1]
        for name in ("k", "v", "ks", "vs"):
            setattr(v, name, [None if t is None else t[b0:b1] for t in getattr(self, name)])
        return v

    def layer_kv(self, layer: int, dtype=None):
        """Dequantised (k, v) of a layer (MLA: latent, None)."""
        dtype = dtype or self.dtype
        if self.kv_dtype == "int8":
            k = dequantize_int8(self.k[layer], self.ks[layer], -1, dtype)
            v = None if self.v[layer] is None else dequantize_int8(self.v[layer], self.vs[layer], -1, dtype)
            return k, v
        return self.k[layer], self.v[layer]

    def nbytes(self) -> int:
        n = 0
        for lst in (self.k, self.v, self.ks, self.vs):
            for t in lst:
                if t is not None:
                    n += t.numel() * t.element_size()
        return n
