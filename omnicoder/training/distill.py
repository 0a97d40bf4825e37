"""Knowledge distillation (reference src/omnicoder/training/distill.py:41-907)
and draft-model / MTP-head training (draft_train.py, speculative_train.py).

loss = alpha * T^2 * KL(softmax(t / T) || softmax(s / T)) + (1 - alpha) * CE(s, labels)
over the vocabulary the two models share (the first min(V_t, V_s) logits).  The
teacher is an omnicoder checkpoint, or a local Hugging Face causal LM directory
(`--teacher_hf`, loaded with local_files_only; nothing is downloaded).

`train_mtp_heads` freezes a trained model and fits its multi-token-prediction
heads (head j predicts token t + 1 + j from the hidden state at t), the
reference's speculative_train; a draft model for speculative decoding is
`distill --student_preset draft_2l`.
"""
from __future__ import annotations

import argparse

import torch
import torch.nn.functional as F


def kd_loss(student_logits, teacher_logits, labels=None, temperature: float = 2.0, alpha: float = 0.9):
    V = min(student_logits.shape[-1], teacher_logits.shape[-1])
    s = student_logits[..., :V].float() / temperature
    t = teacher_logits[..., :V].float() / temperature
    kl = F.kl_div(F.log_softmax(s, -1).reshape(-1, V), F.log_softmax(t, -1).reshape(-1, V), log_target=True,
                  reduction="batchmean") * temperature ** 2
    if labels is None or alpha >= 1.0:
        return kl
    ce = F.cross_entropy(student_logits.float().reshape(-1, student_logits.shape[-1]), labels.reshape(-1),
                         ignore_index=-100)
    return alpha * kl + (1 - alpha) * ce


def _logits(model, ids):
    out = model(ids, all_logits=True) if hasattr(model, "cfg") else model(ids)
    if isinstance(out, dict):
        return out["logits"]
    return out.logits if hasattr(out, "logits") else out[0]


def distill_step(student, teacher, opt, ids, labels, temperature=2.0, alpha=0.9):
    with torch.no_grad():
        t = _logits(teacher, ids)
    s = _logits(student, ids)
    loss = kd_loss(s, t, labels, temperature, alpha)
    loss.backward()
    opt.step()
    opt.zero_grad(set_to_none=True)
    return float(loss)


def train_mtp_heads(model, batches_iter, steps: int, lr: float = 1e-3):
    """Freeze everything except the MTP heads and fit them on `batches_iter`."""
    for p in model.parameters():
        p.requires_grad_(False)
    heads = list(model.mtp_heads)
    for p in heads:
        p.requires_grad_(True)
    opt = torch.optim.AdamW(heads, lr=lr)
    losses = []
    for _ in range(steps):
        ids, lab = next(batches_iter)
        ids, lab = ids.to(heads[0].device), lab.to(heads[0].device)
        with torch.no_grad():
            y, _ = model.hidden(ids)
        B, S = ids.shape
        loss = 0
        for j, w in enumerate(heads):
            logits = (y.float() @ w.float().t()).view(B, S, -1)[:, :S - 1 - j]
            loss = loss + F.cross_entropy(logits.reshape(-1, logits.shape[-1]), lab[:, 1 + j:].reshape(-1))
        loss.backward()
        opt.step()
        opt.zero_grad()
        losses.append(float(loss))
    return losses


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--teacher_ckpt", default=None)
    ap.add_argument("--teacher_preset", default="tiny_moe")
    ap.add_argument("--teacher_hf", default=None, help="local Hugging Face causal LM directory")
    ap.add_argument("--student_preset", default="draft_2l")
    ap.add_argument("--data", default="synthetic")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--seq_len", type=int, default=128)
    ap.add_argument("--batch_size", type=int, default=4)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--temperature", type=float, default=2.0)
    ap.add_argument("--alpha", type=float, default=0.9)
    ap.add_argument("--out", default="weights/student.pt")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    from ..config import get_preset
    from ..inference.builders import load_model
    from ..models.lm import build_model
    from .checkpoint import _atomic_save
    from .data import SyntheticTokens, TextFolderDataset, batches
    dt = torch.float32 if a.device == "cpu" else torch.bfloat16
    if a.teacher_hf:
        from transformers import AutoModelForCausalLM
        teacher = AutoModelForCausalLM.from_pretrained(a.teacher_hf, local_files_only=True).to(a.device).eval()
        vocab = teacher.config.vocab_size
    else:
        teacher = load_model(a.teacher_ckpt, a.device, dtype=dt)[0] if a.teacher_ckpt else \
            build_model(get_preset(a.teacher_preset), a.device, dtype=dt)
        teacher.eval()
        vocab = teacher.cfg.vocab_size
    scfg = get_preset(a.student_preset)
    scfg.vocab_size = vocab
    student = build_model(scfg, a.device, dtype=dt)
    opt = torch.optim.AdamW(student.parameters(), lr=a.lr)
    src = SyntheticTokens(vocab, a.seq_len) if a.data == "synthetic" else TextFolderDataset(a.data, a.seq_len)
    it = batches(src, a.batch_size)
    for step in range(a.steps):
        ids, lab = next(it)
        loss = distill_step(student, teacher, opt, ids.to(a.device), lab.to(a.device), a.temperature, a.alpha)
        print(f"[distill] step {step + 1} loss {loss:.4f}", flush=True)
    _atomic_save({"model": student.state_dict(), "config": student.cfg.to_dict()}, a.out)


if __name__ == "__main__":
    main()
