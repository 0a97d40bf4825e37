"""Decode-time reasoning add-ons (CPU side, off the tensor hot path): self-consistency
voting, tree-of-thoughts MCTS, loopy belief propagation over factor graphs, a
STRIPS-style symbolic planner."""
from .factor_graph import FactorGraph
from .planner import Action, plan
from .search import TreeOfThoughtsMCTS, self_consistency

__all__ = ["FactorGraph", "Action", "plan", "TreeOfThoughtsMCTS", "self_consistency"]
