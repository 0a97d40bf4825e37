"""Preference learning, reward models, uncertainty-shaped rewards and MCTS self-play
(reference src/omnicoder/training/rm_train.py, reward_model.py, rlhf.py,
idk_reward_train.py, mcts_selfplay_rl.py / rl_mcts_selfplay.py).

RewardModel            scalar reward from the final hidden state of a (frozen or trained) LM
reward_pair_loss       Bradley-Terry: -log sigmoid(r_chosen - r_rejected)
train_reward_model     fits the reward head on (prompt+chosen, prompt+rejected) token pairs
PreferenceTrainer      the reference's RLHF objective: a preference loss on the policy's
                       log-probability margins relative to a frozen reference model
                       -log sigmoid(beta * ((pi_c - ref_c) - (pi_r - ref_r))) plus
                       kl_coef * relu(pi_c - ref_c), gradient clipping at 1.0
wrote_idk / reward_idk the uncertainty-shaped reward: +1 correct / -1 wrong, +alpha when a
                       correct answer admits uncertainty, +beta when a wrong one does, and
                       -gamma for a confidently wrong answer
MCTSSelfPlay           self-play on generated arithmetic prompts: a Monte-Carlo tree search
                       over the policy's top next tokens picks a completion, the numeric
                       reward of the searched and of sampled completions drives GRPO updates
"""
from __future__ import annotations

import random
import re
from typing import Callable, Iterable

import torch
import torch.nn as nn
import torch.nn.functional as F

from .rl import GRPOTrainer, completion_logprobs, reward_numeric


# ----------------------------------------------------------------------------
# Reward model
# ----------------------------------------------------------------------------
class RewardModel(nn.Module):
    """r(ids) = head(final normalised hidden state at the last position)."""

    def __init__(self, lm, train_backbone: bool = False):
        super().__init__()
        self.lm = lm
        self.train_backbone = train_backbone
        d = lm.cfg.d_model
        self.head = nn.Sequential(nn.Linear(d, d), nn.GELU(), nn.Linear(d, 1))

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        with torch.set_grad_enabled(self.train_backbone and torch.is_grad_enabled()):
            h, _ = self.lm.hidden(ids)
        last = h.view(ids.shape[0], ids.shape[1], -1)[:, -1].float()
        return self.head(last).squeeze(-1)


def reward_pair_loss(r_chosen: torch.Tensor, r_rejected: torch.Tensor) -> torch.Tensor:
    return -F.logsigmoid(r_chosen - r_rejected).mean()


def train_reward_model(rm: RewardModel, pairs: Iterable, steps: int, lr: float = 1e-4) -> list[float]:
    """pairs yield (chosen ids [B, S], rejected ids [B, S'])."""
    params = [p for p in rm.parameters() if p.requires_grad and (rm.train_backbone or not _in(p, rm.lm))]
    opt = torch.optim.AdamW(params, lr=lr)
    out, it = [], iter(pairs)
    for _ in range(steps):
        ch, rj = next(it)
        loss = reward_pair_loss(rm(ch), rm(rj))
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        out.append(float(loss.detach()))
    return out


def _in(p: torch.Tensor, module: nn.Module) -> bool:
    return any(p is q for q in module.parameters())


# ----------------------------------------------------------------------------
# Preference optimisation against a frozen reference policy
# ----------------------------------------------------------------------------
class PreferenceTrainer:
    def __init__(self, policy, ref, lr: float = 1e-5, beta: float = 1.0, kl_coef: float = 0.05,
                 max_grad_norm: float = 1.0):
        self.policy, self.ref = policy, ref.eval()
        for p in self.ref.parameters():
            p.requires_grad_(False)
        self.opt = torch.optim.AdamW([p for p in policy.parameters() if p.requires_grad], lr=lr)
        self.beta, self.kl_coef, self.max_grad_norm = beta, kl_coef, max_grad_norm

    @staticmethod
    def _seq_logprob(model, ids: torch.Tensor, prompt_len: int) -> torch.Tensor:
        return completion_logprobs(model, ids, max(1, prompt_len)).sum(-1)

    def step(self, chosen: torch.Tensor, rejected: torch.Tensor, prompt_len: int = 1) -> dict:
        """chosen / rejected [B, S] token ids of prompt + response (responses after prompt_len)."""
        with torch.no_grad():
            ref_c = self._seq_logprob(self.ref, chosen, prompt_len)
            ref_r = self._seq_logprob(self.ref, rejected, prompt_len)
        pol_c = self._seq_logprob(self.policy, chosen, prompt_len)
        pol_r = self._seq_logprob(self.policy, rejected, prompt_len)
        margin = (pol_c - ref_c) - (pol_r - ref_r)
        pref = -F.logsigmoid(self.beta * margin).mean()
        kl = torch.relu(pol_c - ref_c).mean()
        loss = pref + self.kl_coef * kl
        loss.backward()
        if self.max_grad_norm > 0:
            torch.nn.utils.clip_grad_norm_(self.policy.parameters(), self.max_grad_norm)
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return {"loss": float(loss.detach()), "pref": float(pref.detach()), "kl": float(kl.detach()),
                "margin": float(margin.detach().mean())}


# ----------------------------------------------------------------------------
# Uncertainty-shaped reward
# ----------------------------------------------------------------------------
_IDK = ("i am not sure", "i'm not sure", "i’m not sure", "i am uncertain", "i don't know", "i do not know")


def wrote_idk(text: str) -> bool:
    t = text.lower()
    return any(p in t for p in _IDK)


def _is_correct(pred: str, gold: str) -> bool:
    p = re.sub(r"\s+", " ", pred.strip().lower())
    g = re.sub(r"\s+", " ", gold.strip().lower())
    return bool(g) and (g in p or p.endswith(g))


def reward_idk(pred: str, gold: str, alpha: float = 0.2, beta: float = 0.3, gamma: float = 0.5) -> float:
    correct = _is_correct(pred, gold)
    idk = wrote_idk(pred)
    r = 1.0 if correct else -1.0
    if idk and correct:
        r += alpha
    elif idk:
        r += beta
    elif not correct:
        r -= gamma
    return r


# ----------------------------------------------------------------------------
# MCTS self-play on arithmetic prompts
# ----------------------------------------------------------------------------
def make_math_prompts(n: int, seed: int = 0, max_operand: int = 50) -> list[tuple[str, int]]:
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        a, b = rng.randint(0, max_operand), rng.randint(0, max_operand)
        op = rng.choice(["+", "-", "*"])
        out.append((f"{a} {op} {b} =", {"+": a + b, "-": a - b, "*": a * b}[op]))
    return out


class MCTSSelfPlay:
    """encode(str) -> list[int], decode(list[int]) -> str.  Each round: for every prompt an MCTS
    over the policy's `branch` most likely next tokens (depth `depth`, leaf value = numeric reward
    of the greedy completion of the leaf) proposes a completion; GRPO then updates the policy on
    sampled groups with the same reward."""

    def __init__(self, policy, encode: Callable, decode: Callable, ref=None, branch: int = 3, depth: int = 3,
                 iterations: int = 24, max_new_tokens: int = 8, lr: float = 1e-5, group: int = 4):
        self.policy, self.encode, self.decode = policy, encode, decode
        self.branch, self.depth, self.iterations, self.max_new = branch, depth, iterations, max_new_tokens
        self.grpo = GRPOTrainer(policy, ref, lr=lr, group=group, max_new_tokens=max_new_tokens)

    @torch.no_grad()
    def _top_tokens(self, ids: list[int]) -> list[int]:
        x = torch.tensor([ids], device=next(self.policy.parameters()).device)
        logits = self.policy(x)["logits"][0, -1].float()
        return logits.topk(self.branch).indices.tolist()

    @torch.no_grad()
    def _rollout_value(self, ids: list[int], target: int) -> float:
        from ..inference.generate import generate
        dev = next(self.policy.parameters()).device
        out = generate(self.policy, torch.tensor([ids], device=dev), self.max_new, temperature=0.0)
        return reward_numeric(self.decode(out[0, len(ids):].tolist()), target)

    def search(self, prompt: str, target: int) -> tuple[str, float]:
        from ..reasoning.search import TreeOfThoughtsMCTS
        base = self.encode(prompt)
        mcts = TreeOfThoughtsMCTS(expand=lambda st: self._top_tokens(base + list(st)),
                                  evaluate=lambda st: self._rollout_value(base + list(st), target),
                                  max_depth=self.depth)
        best = mcts.search((), iterations=self.iterations)
        state = tuple(best.state) if hasattr(best, "state") else tuple(best)
        text = self.decode(list(state))
        return text, self._rollout_value(base + list(state), target)

    def round(self, prompts: list[tuple[str, int]]) -> dict:
        searched = [self.search(p, t)[1] for p, t in prompts]
        enc = [self.encode(p) for p, _ in prompts]
        width = max(len(e) for e in enc)
        dev = next(self.policy.parameters()).device
        ids = torch.tensor([[e[0]] * (width - len(e)) + e for e in enc], device=dev)   # left-pad, equal length
        stats = self.grpo.step(ids, lambda i, comp: reward_numeric(self.decode(comp.tolist()), prompts[i][1]))
        stats["search_reward_mean"] = sum(searched) / max(1, len(searched))
        return stats
