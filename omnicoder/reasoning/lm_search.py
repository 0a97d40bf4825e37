"""Search over a language model's continuations: Tree-of-Thoughts MCTS over next tokens and the
adaptive graph of thoughts over multi-token thoughts (reference
src/omnicoder/reasoning/tot_mcts.py:15-202 -- ToTMCTS(model, tokenizer, cfg).search(prompt) --
and reasoning/adaptive_graph.py:44-476 -- AdaptiveGraphOfThoughts.step(model, ids)).

Both drive the generic searches of omnicoder.reasoning (TreeOfThoughtsMCTS,
AdaptiveGraphOfThoughts) with the model as proposer and evaluator:
  * proposals: the top-k next tokens (MCTS) or k sampled continuations of `thought_len`
    tokens (graph of thoughts);
  * value of a state: the mean log-probability per token of a short greedy rollout under the
    model, or, when the model has a verifier head, the verifier's probability of the last token.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..inference.generate import generate
from .graph_of_thoughts import AdaptiveGraphOfThoughts
from .search import TreeOfThoughtsMCTS


@dataclass
class ToTConfig:
    branch: int = 3           # top-k next tokens expanded per node
    max_depth: int = 4        # tokens added by the search
    iterations: int = 32
    rollout: int = 4          # greedy tokens used to value a leaf
    c: float = 1.4


def _device(model):
    return next(model.parameters()).device


@torch.no_grad()
def _logits(model, ids: list[int]) -> torch.Tensor:
    x = torch.tensor([ids], device=_device(model))
    return model(x, all_logits=True)["logits"][0].float()


@torch.no_grad()
def value_of(model, ids: list[int], rollout: int) -> float:
    """Mean log-probability per token of a greedy rollout after `ids` (or the verifier head's
    probability of the last token when the model has one)."""
    if getattr(model, "verifier", None) is not None:
        x = torch.tensor([ids], device=_device(model))
        y, _ = model.hidden(x)
        v = torch.softmax(y[-1:].float() @ model.verifier.float().t(), -1)[0]
        return float(v[ids[-1]])
    cur, lp = list(ids), 0.0
    for _ in range(rollout):
        logp = torch.log_softmax(_logits(model, cur)[-1], -1)
        t = int(logp.argmax())
        lp += float(logp[t])
        cur.append(t)
    return lp / max(1, rollout)


class LMToTMCTS:
    def __init__(self, model, tokenizer, cfg: ToTConfig | None = None):
        self.model, self.tok, self.cfg = model, tokenizer, cfg or ToTConfig()

    def search(self, prompt: str):
        """-> (best token ids added to the prompt, stats)."""
        base = self.tok.encode(prompt)
        cfg = self.cfg

        def expand(state):
            logp = torch.log_softmax(_logits(self.model, base + list(state))[-1], -1)
            return torch.topk(logp, cfg.branch).indices.tolist()      # actions: the next token

        def evaluate(state):
            return value_of(self.model, base + list(state), cfg.rollout)

        mcts = TreeOfThoughtsMCTS(expand, evaluate, max_depth=cfg.max_depth, c=cfg.c)
        mcts.search((), iterations=cfg.iterations)
        best = list(mcts.best())
        return best, {"iterations": cfg.iterations, "text": self.tok.decode(best)}


class LMAdaptiveGraph:
    """Thoughts are token continuations; each round expands the best frontier thoughts with
    `k` sampled continuations, merges identical ones and keeps the best-valued."""

    def __init__(self, model, tokenizer=None, k: int = 3, thought_len: int = 4, rounds: int = 3, beam: int = 2,
                 temperature: float = 0.8, rollout: int = 2, seed: int = 0):
        self.model, self.tok = model, tokenizer
        self.k, self.L, self.rounds, self.beam, self.temp, self.rollout = k, thought_len, rounds, beam, temperature, \
            rollout
        self.seed = seed

    def step(self, ids: torch.Tensor) -> torch.Tensor:
        """ids [1, S] -> the best continuation found (token ids appended, [1, S + n])."""
        base = ids[0].tolist()
        dev = ids.device
        counter = [self.seed]

        def propose(state):
            x = torch.tensor([base + list(state)], device=dev).repeat(self.k, 1)
            counter[0] += 1
            out = generate(self.model, x, self.L, temperature=self.temp, top_k=0, top_p=1.0, seed=counter[0],
                           cuda_graph=False)
            return [tuple(state) + tuple(o[x.shape[1]:].tolist()) for o in out]

        def score(state):
            return value_of(self.model, base + list(state), self.rollout)

        g = AdaptiveGraphOfThoughts(propose, score, is_final=lambda s: len(s) >= self.L * self.rounds,
                                    key=tuple, beam=self.beam, max_rounds=self.rounds)
        best = g.run(())
        state = best.state if hasattr(best, "state") else best
        return torch.cat([ids, torch.tensor([list(state)], device=dev, dtype=ids.dtype)], 1)
