"""Reinforcement learning from programmatic rewards: GRPO and PPO
(reference src/omnicoder/training/rl_grpo.py:58-835, ppo_rl.py:26-391,
rl_programmatic.py, sfb/runtime/sandbox.py).

GRPO: for every prompt, G completions are sampled; rewards are normalised
within the group, A_i = (r_i - mean) / (std + eps); the loss is
-mean_t[min(rho A, clip(rho, 1 - eps_c, 1 + eps_c) A)] + beta * KL(pi || pi_ref)
with rho = exp(logp - logp_old) over completion tokens and the k3 KL estimator
exp(ref - logp) - (ref - logp) - 1.

PPO: a value head on the final hidden states, the sequence reward on the last
completion token, GAE(gamma, lambda) advantages, clipped policy loss plus a
value loss.

Rewards: exact / normalised match, numeric answer match, substring, and code
execution -- the candidate runs with its tests in a child Python process with a
CPU-time and memory limit and a wall-clock timeout (reward = share of tests
passed).
"""
from __future__ import annotations

import math
import os
import re
import subprocess
import sys
import tempfile

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..inference.generate import generate


# ----------------------------------------------------------------------------
# rewards
# ----------------------------------------------------------------------------
def _norm(s: str) -> str:
    return re.sub(r"\s+", " ", s.strip().lower())


def reward_exact(pred: str, target: str) -> float:
    return 1.0 if _norm(pred) == _norm(target) else 0.0


def reward_contains(pred: str, target: str) -> float:
    return 1.0 if _norm(target) in _norm(pred) else 0.0


def extract_number(s: str):
    m = re.findall(r"-?\d+(?:\.\d+)?", s.replace(",", ""))
    return float(m[-1]) if m else None


def reward_numeric(pred: str, target, tol: float = 1e-6) -> float:
    p = extract_number(pred)
    t = float(target) if not isinstance(target, str) else extract_number(target)
    return 1.0 if (p is not None and t is not None and abs(p - t) <= tol * max(1.0, abs(t))) else 0.0


def run_sandboxed(code: str, timeout_s: float = 5.0, mem_mb: int = 512) -> tuple[int, str]:
    """Run Python `code` in an isolated child process; returns (exit code, output tail)."""
    def limits():
        import resource
        resource.setrlimit(resource.RLIMIT_CPU, (int(timeout_s) + 1, int(timeout_s) + 1))
        resource.setrlimit(resource.RLIMIT_AS, (mem_mb << 20, mem_mb << 20))
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "prog.py")
        with open(path, "w") as f:
            f.write(code)
        try:
            r = subprocess.run([sys.executable, "-I", path], cwd=d, capture_output=True, text=True,
                               timeout=timeout_s, preexec_fn=limits, env={"PATH": "/usr/bin:/bin"})
            return r.returncode, (r.stdout + r.stderr)[-2000:]
        except subprocess.TimeoutExpired:
            return -9, "timeout"


def reward_code(candidate: str, tests: list[str], timeout_s: float = 5.0) -> float:
    if not tests:
        return 0.0
    passed = 0
    for t in tests:
        rc, _ = run_sandboxed(candidate + "\n\n" + t, timeout_s)
        passed += rc == 0
    return passed / len(tests)


# ----------------------------------------------------------------------------
# log-probabilities
# ----------------------------------------------------------------------------
def completion_logprobs(model, ids: torch.Tensor, prompt_len: int) -> torch.Tensor:
    """log p(ids[:, t] | ids[:, :t]) for the completion positions t >= prompt_len -> [B, S - prompt_len]."""
    logits = model(ids[:, :-1], all_logits=True)["logits"].float()
    lp = F.log_softmax(logits, -1).gather(-1, ids[:, 1:, None]).squeeze(-1)
    return lp[:, prompt_len - 1:]


# ----------------------------------------------------------------------------
# GRPO
# ----------------------------------------------------------------------------
class GRPOTrainer:
    def __init__(self, model, ref_model=None, lr: float = 1e-5, group: int = 4, beta: float = 0.02,
                 clip: float = 0.2, max_new_tokens: int = 32, temperature: float = 1.0, top_k: int = 0):
        self.model, self.ref = model, ref_model
        self.opt = torch.optim.AdamW([p for p in model.parameters() if p.requires_grad], lr=lr)
        self.G, self.beta, self.clip = group, beta, clip
        self.max_new, self.temperature, self.top_k = max_new_tokens, temperature, top_k

    def step(self, prompt_ids: torch.Tensor, reward_fn) -> dict:
        """prompt_ids [P, S] (equal-length prompts); reward_fn(prompt index, completion ids) -> float."""
        P, S = prompt_ids.shape
        prompts = prompt_ids.repeat_interleave(self.G, 0)
        self.model.eval()
        with torch.no_grad():
            seqs = generate(self.model, prompts, self.max_new, temperature=self.temperature, top_k=self.top_k,
                            top_p=1.0)
            old_lp = completion_logprobs(self.model, seqs, S)
            ref_lp = completion_logprobs(self.ref, seqs, S) if self.ref is not None else old_lp
        r = torch.tensor([reward_fn(i // self.G, seqs[i, S:]) for i in range(P * self.G)], dtype=torch.float32,
                         device=seqs.device).view(P, self.G)
        adv = ((r - r.mean(1, keepdim=True)) / (r.std(1, keepdim=True, unbiased=False) + 1e-4)).view(-1, 1)
        self.model.train()
        lp = completion_logprobs(self.model, seqs, S)
        rho = torch.exp(lp - old_lp)
        pg = -torch.min(rho * adv, torch.clamp(rho, 1 - self.clip, 1 + self.clip) * adv)
        kl = torch.exp(ref_lp - lp) - (ref_lp - lp) - 1
        loss = (pg + self.beta * kl).mean()
        loss.backward()
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return {"loss": float(loss), "reward_mean": float(r.mean()), "kl": float(kl.mean())}


# ----------------------------------------------------------------------------
# PPO
# ----------------------------------------------------------------------------
class ValueHead(nn.Module):
    def __init__(self, d_model: int):
        super().__init__()
        self.v = nn.Linear(d_model, 1)

    def forward(self, h):
        return self.v(h.float()).squeeze(-1)


def gae(rewards: torch.Tensor, values: torch.Tensor, gamma: float = 1.0, lam: float = 0.95):
    """rewards, values [B, T] -> (advantages, returns)."""
    B, T = rewards.shape
    adv = torch.zeros_like(rewards)
    last = torch.zeros(B, device=rewards.device)
    for t in range(T - 1, -1, -1):
        nv = values[:, t + 1] if t + 1 < T else torch.zeros(B, device=rewards.device)
        delta = rewards[:, t] + gamma * nv - values[:, t]
        last = delta + gamma * lam * last
        adv[:, t] = last
    return adv, adv + values


class PPOTrainer:
    def __init__(self, model, lr: float = 1e-5, clip: float = 0.2, vf_coef: float = 0.5, max_new_tokens: int = 32,
                 temperature: float = 1.0, gamma: float = 1.0, lam: float = 0.95):
        self.model = model
        dev = next(model.parameters()).device
        self.value = ValueHead(model.cfg.d_model).to(dev)
        self.opt = torch.optim.AdamW(list(p for p in model.parameters() if p.requires_grad) +
                                     list(self.value.parameters()), lr=lr)
        self.clip, self.vf, self.max_new, self.temperature, self.gamma, self.lam = clip, vf_coef, max_new_tokens, \
            temperature, gamma, lam

    def _lp_values(self, seqs, S):
        y, _ = self.model.hidden(seqs[:, :-1])
        B, L = seqs.shape
        logits = (y.float() @ self.model.head_weight.float().t()).view(B, L - 1, -1)
        lp = F.log_softmax(logits, -1).gather(-1, seqs[:, 1:, None]).squeeze(-1)[:, S - 1:]
        v = self.value(y.view(B, L - 1, -1))[:, S - 1:]
        return lp, v

    def step(self, prompt_ids: torch.Tensor, reward_fn) -> dict:
        S = prompt_ids.shape[1]
        self.model.eval()
        with torch.no_grad():
            seqs = generate(self.model, prompt_ids, self.max_new, temperature=self.temperature, top_k=0, top_p=1.0)
            old_lp, old_v = self._lp_values(seqs, S)
            r = torch.tensor([reward_fn(i, seqs[i, S:]) for i in range(seqs.shape[0])], dtype=torch.float32,
                             device=seqs.device)
            tok_r = torch.zeros_like(old_lp)
            tok_r[:, -1] = r
            adv, ret = gae(tok_r, old_v.float(), self.gamma, self.lam)
            adv = (adv - adv.mean()) / (adv.std() + 1e-6)
        self.model.train()
        lp, v = self._lp_values(seqs, S)
        rho = torch.exp(lp - old_lp)
        pol = -torch.min(rho * adv, torch.clamp(rho, 1 - self.clip, 1 + self.clip) * adv).mean()
        vl = F.mse_loss(v.float(), ret)
        loss = pol + self.vf * vl
        loss.backward()
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return {"loss": float(loss), "policy": float(pol), "value": float(vl), "reward_mean": float(r.mean())}


# ----------------------------------------------------------------------------
# CLI: python -m omnicoder.training.rl
# ----------------------------------------------------------------------------
def arithmetic_prompts(n: int, seed: int = 0) -> list[dict]:
    """Programmatic tasks with checkable answers: "a + b =" / "a * b =" with small operands."""
    import random
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        a, b = rng.randint(0, 20), rng.randint(0, 20)
        op = rng.choice("+*")
        out.append({"prompt": f"{a} {op} {b} =", "answer": a + b if op == "+" else a * b})
    return out


def main(argv=None):
    import argparse
    import json

    from ..config import get_preset
    from ..models.lm import build_model
    from .tokenizer import get_tokenizer
    ap = argparse.ArgumentParser(description="GRPO / PPO with programmatic rewards")
    ap.add_argument("--algo", default="grpo", choices=["grpo", "ppo"])
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--ckpt", default="")
    ap.add_argument("--prompts", default="", help="JSONL {prompt, answer} (default: arithmetic tasks)")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--batch", type=int, default=2, help="prompts per step")
    ap.add_argument("--group", type=int, default=4)
    ap.add_argument("--max_new_tokens", type=int, default=8)
    ap.add_argument("--lr", type=float, default=1e-5)
    ap.add_argument("--out", default="weights/rl.pt")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    if a.ckpt:
        from ..inference.builders import load_model
        model, _ = load_model(a.ckpt, a.device, dtype=torch.float32, preset=a.preset)
    else:
        model = build_model(get_preset(a.preset), device=a.device, dtype=torch.float32, seed=0)
    tok = get_tokenizer(model.cfg.vocab_size)
    tasks = ([json.loads(l) for l in open(a.prompts) if l.strip()] if a.prompts else arithmetic_prompts(64))
    if a.algo == "grpo":
        tr = GRPOTrainer(model, lr=a.lr, group=a.group, max_new_tokens=a.max_new_tokens)
    else:
        tr = PPOTrainer(model, lr=a.lr, max_new_tokens=a.max_new_tokens)
    hist = []
    for s in range(a.steps):
        batch = [tasks[(s * a.batch + i) % len(tasks)] for i in range(a.batch)]
        enc = [tok.encode(t["prompt"]) for t in batch]
        L = max(len(e) for e in enc)
        ids = torch.tensor([[0] * (L - len(e)) + e for e in enc], device=a.device)   # left-pad to one length
        rfn = lambda i, comp, batch=batch: reward_numeric(tok.decode(comp.tolist()), batch[i]["answer"])
        hist.append(tr.step(ids, rfn))
    torch.save({"model": model.export_state_dict(), "config": model.cfg.to_dict(), "step": a.steps}, a.out)
    print(json.dumps({"steps": a.steps, "last": hist[-1] if hist else None, "out": a.out}))
    return 0


if __name__ == "__main__":
    main()
