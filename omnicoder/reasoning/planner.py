"""STRIPS-style symbolic planning (reference src/omnicoder/reasoning/symbolic_planner.py:1-154):
states are sets of facts, actions have preconditions, add and delete lists;
breadth-first search returns a shortest action sequence reaching the goal."""
from __future__ import annotations

import collections
from dataclasses import dataclass, field


@dataclass(frozen=True)
class Action:
    name: str
    pre: frozenset = field(default_factory=frozenset)
    add: frozenset = field(default_factory=frozenset)
    delete: frozenset = field(default_factory=frozenset)


def plan(initial, goal, actions: list[Action], max_depth: int = 32) -> list[str] | None:
    start, goal = frozenset(initial), frozenset(goal)
    q = collections.deque([(start, [])])
    seen = {start}
    while q:
        s, path = q.popleft()
        if goal <= s:
            return path
        if len(path) >= max_depth:
            continue
        for a in actions:
            if a.pre <= s:
                n = (s - a.delete) | a.add
                if n not in seen:
                    seen.add(n)
                    q.append((n, path + [a.name]))
    return None
