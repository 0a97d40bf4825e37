"""Search over generations (reference src/omnicoder/reasoning/tot_mcts.py:1-202,
adaptive_graph.py, omega_controller.py).

self_consistency: sample n answers, return the most frequent extracted answer
and its vote share.
TreeOfThoughtsMCTS: nodes are partial solutions (lists of "thoughts");
`expand(state) -> [thought, ...]` proposes children, `evaluate(state) ->
value in [0, 1]` scores leaves; selection by UCT (mean value + c * sqrt(ln N /
n)), one expansion and one evaluation per iteration, values backed up along
the path.  `best()` returns the most visited path.
"""
from __future__ import annotations

import collections
import math
from typing import Callable


def self_consistency(sample_fn: Callable[[], str], n: int = 8, extract: Callable[[str], str] = str.strip):
    votes = collections.Counter(extract(sample_fn()) for _ in range(n))
    ans, c = votes.most_common(1)[0]
    return ans, c / n


class _Node:
    __slots__ = ("state", "parent", "children", "n", "w", "untried")

    def __init__(self, state, parent=None):
        self.state, self.parent = state, parent
        self.children: list[_Node] = []
        self.n, self.w = 0, 0.0
        self.untried = None


class TreeOfThoughtsMCTS:
    def __init__(self, expand: Callable, evaluate: Callable, max_depth: int = 4, c: float = 1.4):
        self.expand, self.evaluate, self.max_depth, self.c = expand, evaluate, max_depth, c

    def _uct(self, child, parent_n):
        return child.w / child.n + self.c * math.sqrt(math.log(parent_n) / child.n)

    def search(self, root_state=(), iterations: int = 64):
        self.root = _Node(tuple(root_state))
        for _ in range(iterations):
            node = self.root
            while node.untried is not None and not node.untried and node.children:
                node = max(node.children, key=lambda ch: self._uct(ch, node.n))
            if node.untried is None:
                node.untried = list(self.expand(node.state)) if len(node.state) < self.max_depth else []
            if node.untried:
                t = node.untried.pop(0)
                child = _Node(node.state + (t,), node)
                node.children.append(child)
                node = child
            value = float(self.evaluate(node.state))
            while node is not None:
                node.n += 1
                node.w += value
                node = node.parent
        return self.best()

    def best(self):
        node, path = self.root, []
        while node.children:
            node = max(node.children, key=lambda ch: ch.n)
            path = node.state
        return list(path)
