"""Evaluation: perplexity, exact-match / numeric accuracy, pass@k on code tasks, throughput."""
from .metrics import auto_benchmark, evaluate_code, evaluate_qa, pass_at_k, perplexity

__all__ = ["auto_benchmark", "evaluate_code", "evaluate_qa", "pass_at_k", "perplexity"]
