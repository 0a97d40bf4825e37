"""Image and video generation through the language model's unified vocabulary.

The reference generates images and videos with external diffusion pipelines
(src/omnicoder/modeling/multimodal/image_pipeline.py:1-345, video_pipeline.py:1-373,
weights downloaded from a hub) and also defines the unified token layout in
which the model itself can emit image / video codebook ids
(src/omnicoder/modeling/multimodal/vocab_map.py:12-169).  This module runs the
second path with no external weights: the model samples a grid of code tokens
autoregressively (after the prompt, with its KV cache), every step restricted to
the modality's id range of the unified vocabulary, and the codes are decoded to
pixels by the VQ-VAE decoder of that modality.

    generate_codes(model, prompt, lo, n_codes, count, ...)   -> codes [B, count] in [0, n_codes)
    generate_image(model, vq, prompt, vocab, grid=(h, w))    -> images [B, 3, H, W] in [0, 1]
    generate_video(model, vq, prompt, vocab, frames, grid)   -> videos [B, T, 3, H, W] in [0, 1]
"""
from __future__ import annotations

import torch


@torch.no_grad()
def generate_codes(model, prompt: torch.Tensor, lo: int, n_codes: int, count: int, temperature: float = 1.0,
                   top_k: int = 0, generator: torch.Generator | None = None) -> torch.Tensor:
    """Sample `count` tokens after `prompt` [B, S], each from ids [lo, lo + n_codes) only;
    returns them shifted to [0, n_codes)."""
    from ..inference.kv_cache import KVCache
    if lo + n_codes > model.cfg.vocab_size:
        raise ValueError(f"code range [{lo}, {lo + n_codes}) exceeds the model vocabulary ({model.cfg.vocab_size})")
    B, S = prompt.shape
    dev = prompt.device
    cache = KVCache(model.cfg, B, S + count, dev)
    logits = model.forward_cached(prompt, cache, prefill=True, last_only=True)[:, -1]
    out = torch.empty(B, count, dtype=torch.long, device=dev)
    for i in range(count):
        z = logits[:, lo:lo + n_codes].float()
        if temperature <= 0:
            code = z.argmax(-1)
        else:
            z = z / temperature
            if 0 < top_k < n_codes:
                kth = z.topk(top_k, dim=-1).values[:, -1:]
                z = z.masked_fill(z < kth, float("-inf"))
            code = torch.multinomial(torch.softmax(z, -1), 1, generator=generator).squeeze(1)
        out[:, i] = code
        if i + 1 < count:
            logits = model.forward_cached((code + lo).view(B, 1), cache)[:, -1]
    return out


def _range(vocab, name: str) -> tuple[int, int]:
    a, b = getattr(vocab, f"{name}_range")
    return a, b - a + 1


@torch.no_grad()
def generate_image(model, vq, prompt: torch.Tensor, vocab, grid: tuple[int, int] = (16, 16), **sample) -> torch.Tensor:
    lo, n = _range(vocab, "image")
    K = vq.vq.codebook.num_embeddings
    h, w = grid
    codes = generate_codes(model, prompt, lo, min(n, K), h * w, **sample)
    img = vq.decode(codes.view(-1, h, w).to(next(vq.parameters()).device))
    return img.clamp(0, 1)


@torch.no_grad()
def generate_video(model, vq, prompt: torch.Tensor, vocab, frames: int = 4, grid: tuple[int, int] = (8, 8),
                   **sample) -> torch.Tensor:
    lo, n = _range(vocab, "video")
    K = vq.image.vq.codebook.num_embeddings
    h, w = grid
    codes = generate_codes(model, prompt, lo, min(n, K), frames * h * w, **sample)
    vid = vq.decode(codes.view(-1, frames, h, w).to(next(vq.parameters()).device))
    return vid.clamp(0, 1)
