"""Code-expert pretraining: distillation on code with router-distribution distillation and
balanced expert assignment (reference src/omnicoder/training/code_expert_pretrain.py, which
configures the distillation run with router KD and Sinkhorn-balanced routing to specialise experts
to code without destabilising routing).

Loss per batch (student S, teacher T, both MoE LMs; the router terms need the same expert count):

  kd_loss(S, T)                                                   (logit distillation, distill.py)
  + router_kd * mean over MoE layers of KL(p_T || p_S)            p = softmax(y W_router^T) per token
  + balance  * mean over layers of CE(sinkhorn(z_S), log softmax(z_S))

sinkhorn(z) alternately normalises exp(z) over experts and over tokens (equal expert loads), the
balanced-assignment target; its cross entropy pulls each token's routing towards an assignment in
which every expert receives the same share of tokens.  Router inputs are captured with forward hooks
on the MoE layers (the router logits are recomputed from them: one [T, D] x [D, E] product per layer).
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.nn.functional as F

from .distill import kd_loss


def sinkhorn(logits: torch.Tensor, iters: int = 3) -> torch.Tensor:
    """[T, E] logits -> assignment with rows summing to 1 and columns to T / E."""
    T, E = logits.shape
    p = torch.softmax(logits.float() - logits.float().max(), -1)
    for _ in range(iters):
        p = p / p.sum(0, keepdim=True).clamp_min(1e-12) * (T / E)     # equal expert loads
        p = p / p.sum(1, keepdim=True).clamp_min(1e-12)                # one unit per token
    return p


class RouterTap:
    """Captures the input of every MoE layer's router during a forward pass."""

    def __init__(self, model):
        from ..models.lm import MoEFFN
        self.layers = [m for m in model.modules() if isinstance(m, MoEFFN)]
        self.inputs: list = [None] * len(self.layers)
        self._h = [m.register_forward_hook(self._hook(i)) for i, m in enumerate(self.layers)]

    def _hook(self, i):
        def f(module, inp, out):
            self.inputs[i] = inp[0]
        return f

    def logits(self) -> list[torch.Tensor]:
        return [x.reshape(-1, x.shape[-1]).float() @ m.router.float().t()
                for x, m in zip(self.inputs, self.layers) if x is not None]

    def close(self):
        for h in self._h:
            h.remove()


def _logits(model, ids):
    out = model(ids, all_logits=True)
    return out["logits"] if isinstance(out, dict) else out


def code_expert_loss(student, teacher, s_tap: RouterTap, t_tap: RouterTap | None, ids, labels,
                     temperature: float = 2.0, alpha: float = 0.9, router_kd: float = 0.1,
                     balance: float = 0.01) -> tuple[torch.Tensor, dict]:
    with torch.no_grad():
        t_logits = _logits(teacher, ids)
    s_logits = _logits(student, ids)
    loss = kd_loss(s_logits, t_logits, labels, temperature, alpha)
    parts = {"kd": float(loss.detach())}
    zs = s_tap.logits()
    if router_kd > 0 and t_tap is not None:
        zt = [z.detach() for z in t_tap.logits()]
        pairs = [(a, b) for a, b in zip(zs, zt) if a.shape == b.shape]
        if pairs:
            rk = sum(F.kl_div(F.log_softmax(a, -1), F.log_softmax(b, -1), log_target=True, reduction="batchmean")
                     for a, b in pairs) / len(pairs)
            loss = loss + router_kd * rk
            parts["router_kd"] = float(rk.detach())
    if balance > 0 and zs:
        bal = sum(-(sinkhorn(z.detach()) * F.log_softmax(z, -1)).sum(-1).mean() for z in zs) / len(zs)
        loss = loss + balance * bal
        parts["balance"] = float(bal.detach())
    return loss, parts


def main(argv=None):
    from ..config import get_preset
    from ..inference.builders import load_model
    from ..models.lm import build_model
    from .checkpoint import _atomic_save
    from .data import SyntheticTokens, TextFolderDataset, batches
    ap = argparse.ArgumentParser(description="code-expert distillation with router KD and balanced routing")
    ap.add_argument("--data", default="synthetic", help="folder of code files (default: synthetic tokens)")
    ap.add_argument("--teacher_ckpt", default=None)
    ap.add_argument("--teacher_preset", default="tiny_moe")
    ap.add_argument("--student_preset", default="tiny_moe")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--seq_len", type=int, default=128)
    ap.add_argument("--batch_size", type=int, default=2)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--temperature", type=float, default=2.0)
    ap.add_argument("--alpha", type=float, default=0.9)
    ap.add_argument("--router_kd", type=float, default=0.1)
    ap.add_argument("--balance", type=float, default=0.01)
    ap.add_argument("--out", default="weights/code_expert.pt")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dt = torch.float32 if a.device == "cpu" else torch.bfloat16
    teacher = (load_model(a.teacher_ckpt, a.device, dtype=dt)[0] if a.teacher_ckpt else
               build_model(get_preset(a.teacher_preset), a.device, dtype=dt, seed=1)).eval()
    scfg = get_preset(a.student_preset)
    scfg.vocab_size = teacher.cfg.vocab_size
    student = build_model(scfg, a.device, dtype=dt, seed=0)
    s_tap, t_tap = RouterTap(student), RouterTap(teacher)
    opt = torch.optim.AdamW(student.parameters(), lr=a.lr)
    src = SyntheticTokens(scfg.vocab_size, a.seq_len) if a.data == "synthetic" else \
        TextFolderDataset(a.data, a.seq_len)
    it = batches(src, a.batch_size)
    log = []
    for _ in range(a.steps):
        ids, lab = next(it)
        ids, lab = ids.to(a.device), lab.to(a.device)
        loss, parts = code_expert_loss(student, teacher, s_tap, t_tap, ids, lab, a.temperature, a.alpha,
                                       a.router_kd, a.balance)
        opt.zero_grad(set_to_none=True)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(student.parameters(), 1.0)
        opt.step()
        log.append(parts)
    s_tap.close()
    t_tap.close()
    _atomic_save({"model": student.export_state_dict(), "config": student.cfg.to_dict()}, a.out)
    print(json.dumps({"steps": a.steps, "first": log[0] if log else None, "last": log[-1] if log else None,
                      "out": a.out}))
    return 0


if __name__ == "__main__":
    main()
