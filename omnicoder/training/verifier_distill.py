"""Verifier-head distillation (reference src/omnicoder/training/verifier_distill.py:41-268).

The verifier head scores the next token at every position; speculative decoding accepts a
draft token when the verifier's probability of it clears a threshold (generate(...,
verify_threshold=)).  It is trained to match a teacher's softened next-token distribution:

    loss = KL(teacher_T || student_T) * (0 if verifier_only else 1) + KL(teacher_T || verifier_T)

with both distributions at temperature `kl_temp` (the reference's two KL terms, batch-mean over
positions, gradient-norm clip 1.0).  When the teacher's vocabulary differs from the student's
(a local Hugging Face teacher), a learned linear map from student to teacher logits is trained
jointly, as in the reference.  Unlike the reference, whose verifier reads the token embeddings,
the verifier here reads the final-norm hidden state, the same input as the LM head; that is
what decoding uses it on.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.nn as nn
import torch.nn.functional as F


def _teacher_logits(teacher, ids: torch.Tensor) -> torch.Tensor:
    with torch.no_grad():
        out = teacher(ids, all_logits=True) if hasattr(teacher, "cfg") else teacher(ids)
    if isinstance(out, dict):
        return out["logits"]
    return out.logits if hasattr(out, "logits") else out[0]


def student_and_verifier_logits(student, ids: torch.Tensor):
    """(LM-head logits, verifier logits) [B, S, V] from one pass of the student."""
    y, _ = student.hidden(ids)
    B, S = ids.shape
    return ((y @ student.head_weight.t()).view(B, S, -1).float(), (y @ student.verifier.t()).view(B, S, -1).float())


class VerifierDistiller:
    def __init__(self, student, lr: float = 2e-4, kl_temp: float = 1.5, verifier_only: bool = False,
                 teacher_vocab: int | None = None):
        if getattr(student, "verifier", None) is None:
            raise ValueError("the student has no verifier head (ModelConfig.verifier_head)")
        self.student, self.temp, self.verifier_only = student, kl_temp, verifier_only
        if verifier_only:
            for n, p in student.named_parameters():
                p.requires_grad_(n == "verifier")
        V = student.cfg.vocab_size
        self.align = None
        if teacher_vocab is not None and teacher_vocab != V:
            dev = student.verifier.device
            self.align = nn.Linear(V, teacher_vocab, bias=False, device=dev, dtype=torch.float32)
        params = [p for p in student.parameters() if p.requires_grad]
        if self.align is not None:
            params += list(self.align.parameters())
        self.opt = torch.optim.AdamW(params, lr=lr)

    def loss(self, ids: torch.Tensor, t_logits: torch.Tensor) -> torch.Tensor:
        s_logits, v_logits = student_and_verifier_logits(self.student, ids)
        if self.align is not None:
            s_logits, v_logits = self.align(s_logits), self.align(v_logits)
        T = max(1e-6, self.temp)
        t = F.log_softmax(t_logits.float() / T, -1).reshape(-1, t_logits.shape[-1])
        kl = lambda x: F.kl_div(F.log_softmax(x / T, -1).reshape(-1, x.shape[-1]), t, log_target=True,
                                reduction="batchmean")
        loss = kl(v_logits)
        if not self.verifier_only:
            loss = loss + kl(s_logits)
        return loss

    def step(self, ids: torch.Tensor, t_logits: torch.Tensor) -> float:
        loss = self.loss(ids, t_logits)
        self.opt.zero_grad(set_to_none=True)
        loss.backward()
        params = [p for g in self.opt.param_groups for p in g["params"]]
        torch.nn.utils.clip_grad_norm_(params, 1.0)
        self.opt.step()
        return float(loss.detach())


def main(argv=None):
    from ..config import get_preset
    from ..inference.builders import load_model
    from ..models.lm import build_model
    from .checkpoint import _atomic_save
    from .data import SyntheticTokens, TextFolderDataset, batches
    ap = argparse.ArgumentParser(description="verifier-head distillation")
    ap.add_argument("--data", default="synthetic", help="text folder (default: synthetic tokens)")
    ap.add_argument("--seq_len", type=int, default=128)
    ap.add_argument("--batch_size", type=int, default=2)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--student_preset", default="tiny_moe")
    ap.add_argument("--load_student", default="", help="student checkpoint to start from")
    ap.add_argument("--teacher_ckpt", default=None)
    ap.add_argument("--teacher_preset", default="tiny_moe")
    ap.add_argument("--teacher_hf", default=None, help="local Hugging Face causal LM directory")
    ap.add_argument("--lr", type=float, default=2e-4)
    ap.add_argument("--kl_temp", type=float, default=1.5)
    ap.add_argument("--verifier_only", action="store_true", help="update only the verifier head")
    ap.add_argument("--out", default="weights/omnicoder_verifier_kd.pt")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dt = torch.float32 if a.device == "cpu" else torch.bfloat16
    if a.teacher_hf:
        from transformers import AutoModelForCausalLM
        teacher = AutoModelForCausalLM.from_pretrained(a.teacher_hf, local_files_only=True).to(a.device).eval()
        tvocab = teacher.config.vocab_size
    else:
        teacher = (load_model(a.teacher_ckpt, a.device, dtype=dt)[0] if a.teacher_ckpt else
                   build_model(get_preset(a.teacher_preset), a.device, dtype=dt, seed=1)).eval()
        tvocab = teacher.cfg.vocab_size
    if a.load_student:
        student = load_model(a.load_student, a.device, dtype=dt)[0]
    else:
        cfg = get_preset(a.student_preset)
        cfg.verifier_head = True
        student = build_model(cfg, a.device, dtype=dt, seed=0)
    if getattr(student, "verifier", None) is None:
        raise SystemExit("the student checkpoint has no verifier head")
    vd = VerifierDistiller(student, a.lr, a.kl_temp, a.verifier_only, teacher_vocab=tvocab)
    src = SyntheticTokens(student.cfg.vocab_size, a.seq_len) if a.data == "synthetic" else \
        TextFolderDataset(a.data, a.seq_len)
    it = batches(src, a.batch_size)
    losses = []
    for _ in range(a.steps):
        ids, _lab = next(it)
        ids = ids.to(a.device)
        losses.append(vd.step(ids, _teacher_logits(teacher, ids)))
    _atomic_save({"model": student.export_state_dict(), "config": student.cfg.to_dict(),
                  "align": None if vd.align is None else vd.align.state_dict()}, a.out)
    print(json.dumps({"steps": a.steps, "first_loss": losses[0] if losses else None,
                      "last_loss": losses[-1] if losses else None, "out": a.out}))
    return 0


if __name__ == "__main__":
    main()
