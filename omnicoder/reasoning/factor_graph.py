"""Discrete factor graphs with loopy belief propagation (sum-product)
(reference src/omnicoder/sfb/inference/bp.py, factor_graph.py:1-365).

Variables have finite domains; factors are non-negative tables over a tuple of
variables.  `marginals(iters, damping)` runs synchronous message passing
(variable->factor and factor->variable, normalised, optionally damped) and
returns per-variable marginals; on trees it is exact.  `exact_marginals()`
enumerates the joint (small graphs; the tests' oracle).
"""
from __future__ import annotations

import itertools

import numpy as np


class FactorGraph:
    def __init__(self):
        self.card: dict[str, int] = {}
        self.factors: list[tuple[tuple[str, ...], np.ndarray]] = []

    def add_variable(self, name: str, card: int) -> None:
        self.card[name] = card

    def add_factor(self, variables: tuple[str, ...], table) -> None:
        t = np.asarray(table, dtype=np.float64)
        assert t.shape == tuple(self.card[v] for v in variables), "factor table shape"
        self.factors.append((tuple(variables), t))

    def marginals(self, iters: int = 50, damping: float = 0.0) -> dict[str, np.ndarray]:
        f2v = {(i, v): np.ones(self.card[v]) / self.card[v] for i, (vs, _) in enumerate(self.factors) for v in vs}
        v2f = dict(f2v)
        for _ in range(iters):
            for (i, v) in v2f:
                m = np.ones(self.card[v])
                for (j, w), msg in f2v.items():
                    if w == v and j != i:
                        m = m * msg
                v2f[(i, v)] = m / m.sum()
            new = {}
            for i, (vs, t) in enumerate(self.factors):
                for k, v in enumerate(vs):
                    x = t.copy()
                    for kk, w in enumerate(vs):
                        if kk != k:
                            shape = [1] * len(vs)
                            shape[kk] = self.card[w]
                            x = x * v2f[(i, w)].reshape(shape)
                    m = x.sum(axis=tuple(kk for kk in range(len(vs)) if kk != k))
                    m = m / m.sum()
                    new[(i, v)] = damping * f2v[(i, v)] + (1 - damping) * m
            f2v = new
        out = {}
        for v in self.card:
            b = np.ones(self.card[v])
            for (i, w), msg in f2v.items():
                if w == v:
                    b = b * msg
            out[v] = b / b.sum()
        return out

    def exact_marginals(self) -> dict[str, np.ndarray]:
        names = list(self.card)
        joint = np.zeros([self.card[v] for v in names])
        for assign in itertools.product(*[range(self.card[v]) for v in names]):
            a = dict(zip(names, assign))
            p = 1.0
            for vs, t in self.factors:
                p *= t[tuple(a[v] for v in vs)]
            joint[assign] = p
        joint /= joint.sum()
        return {v: joint.sum(axis=tuple(j for j in range(len(names)) if j != i)) for i, v in enumerate(names)}
