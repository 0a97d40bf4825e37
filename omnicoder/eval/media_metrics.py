"""Evaluation metrics for text, image, audio and video outputs
(reference src/omnicoder/eval/text_eval.py, image_eval.py, audio_eval.py,
video_eval.py, reward_metrics.py, auto_benchmark.py:163-230; those call external
CLIP / FID / FAD / ASR packages, which are not dependencies here: the
distribution metrics take features from whatever encoder the caller supplies).

word_error_rate      word-level Levenshtein distance / reference length
bleu                 corpus BLEU (modified n-gram precision up to n=4, brevity penalty)
exact_match_accuracy normalised string equality over (prediction, answer) pairs
psnr                 10 log10(max^2 / MSE)
ssim                 structural similarity with an 11-tap Gaussian window (sigma 1.5),
                     constants (0.01 L)^2 and (0.03 L)^2 (Wang et al., 2004)
frechet_distance     |mu1 - mu2|^2 + Tr(S1 + S2 - 2 (S1 S2)^(1/2)) between two feature sets
                     (FID / FAD / FVD given image, audio or video features)
embedding_alignment  mean cosine similarity of paired embeddings (a CLIP-score style measure
                     for any pair of encoders)
temporal_consistency mean cosine similarity of consecutive frame features of a video
snr_db               10 log10(|ref|^2 / |ref - est|^2)
"""
from __future__ import annotations

import math
import re
from collections import Counter

import numpy as np
import torch
import torch.nn.functional as F


def _edit(a: list, b: list) -> int:
    prev = list(range(len(b) + 1))
    for i, x in enumerate(a, 1):
        cur = [i]
        for j, y in enumerate(b, 1):
            cur.append(min(prev[j] + 1, cur[j - 1] + 1, prev[j - 1] + (x != y)))
        prev = cur
    return prev[-1]


def word_error_rate(reference: str, hypothesis: str) -> float:
    ref, hyp = reference.split(), hypothesis.split()
    return _edit(ref, hyp) / max(1, len(ref))


def _ngrams(words: list[str], n: int) -> Counter:
    return Counter(tuple(words[i:i + n]) for i in range(len(words) - n + 1))


def bleu(predictions: list[str], references: list[list[str]], max_n: int = 4) -> float:
    match = [0] * max_n
    total = [0] * max_n
    hyp_len = ref_len = 0
    for pred, refs in zip(predictions, references):
        p = pred.split()
        rs = [r.split() for r in refs]
        hyp_len += len(p)
        ref_len += min((abs(len(r) - len(p)), len(r)) for r in rs)[1]
        for n in range(1, max_n + 1):
            pc = _ngrams(p, n)
            best = Counter()
            for r in rs:
                best |= _ngrams(r, n)
            match[n - 1] += sum(min(c, best[g]) for g, c in pc.items())
            total[n - 1] += max(0, len(p) - n + 1)
    if hyp_len == 0 or min(match) == 0:
        return 0.0
    logp = sum(math.log(m / t) for m, t in zip(match, total)) / max_n
    bp = 1.0 if hyp_len > ref_len else math.exp(1 - ref_len / hyp_len)
    return bp * math.exp(logp)


def _norm(s: str) -> str:
    return re.sub(r"\s+", " ", re.sub(r"[^\w\s]", "", s.lower())).strip()


def exact_match_accuracy(pairs: list[tuple[str, str]]) -> float:
    return sum(_norm(p) == _norm(a) for p, a in pairs) / max(1, len(pairs))


def psnr(pred: torch.Tensor, target: torch.Tensor, max_val: float = 1.0) -> float:
    mse = F.mse_loss(pred.float(), target.float()).item()
    return float("inf") if mse == 0 else 10 * math.log10(max_val ** 2 / mse)


def _gauss(size: int = 11, sigma: float = 1.5) -> torch.Tensor:
    x = torch.arange(size, dtype=torch.float32) - size // 2
    g = torch.exp(-x * x / (2 * sigma * sigma))
    return g / g.sum()


def ssim(pred: torch.Tensor, target: torch.Tensor, max_val: float = 1.0) -> float:
    """pred, target [B, C, H, W]; mean SSIM over the valid window positions."""
    x, y = pred.float(), target.float()
    C = x.shape[1]
    g = _gauss().to(x.device)
    w = (g[:, None] * g[None, :]).expand(C, 1, 11, 11).contiguous()
    f = lambda t: F.conv2d(t, w, groups=C)
    mx, my = f(x), f(y)
    sxx, syy, sxy = f(x * x) - mx * mx, f(y * y) - my * my, f(x * y) - mx * my
    c1, c2 = (0.01 * max_val) ** 2, (0.03 * max_val) ** 2
    m = ((2 * mx * my + c1) * (2 * sxy + c2)) / ((mx * mx + my * my + c1) * (sxx + syy + c2))
    return float(m.mean())


def frechet_distance(feats_a: torch.Tensor, feats_b: torch.Tensor) -> float:
    from scipy import linalg
    a = feats_a.double().cpu().numpy()
    b = feats_b.double().cpu().numpy()
    mu1, mu2 = a.mean(0), b.mean(0)
    s1, s2 = np.cov(a, rowvar=False), np.cov(b, rowvar=False)
    covmean = np.real(linalg.sqrtm(s1 @ s2))
    return float(((mu1 - mu2) ** 2).sum() + np.trace(s1 + s2 - 2 * covmean))


def embedding_alignment(emb_a: torch.Tensor, emb_b: torch.Tensor) -> float:
    return float(F.cosine_similarity(emb_a.float(), emb_b.float(), dim=-1).mean())


def temporal_consistency(frame_feats: torch.Tensor) -> float:
    """frame_feats [T, D] or [B, T, D]."""
    f = frame_feats.float()
    return float(F.cosine_similarity(f[..., 1:, :], f[..., :-1, :], dim=-1).mean())


def snr_db(reference: torch.Tensor, estimate: torch.Tensor) -> float:
    r = reference.float()
    noise = (r - estimate.float()).pow(2).sum().item()
    return float("inf") if noise == 0 else 10 * math.log10(r.pow(2).sum().item() / noise)
