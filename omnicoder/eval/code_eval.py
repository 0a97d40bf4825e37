"""Functional-correctness evaluation of generated code (reference src/omnicoder/eval/code_eval.py:1-40).

The candidate is written to ``sol.py`` in a fresh temporary folder, the task's tests to ``test.py`` beside it
(so tests may ``from sol import ...``), and ``test.py`` runs in a child interpreter under the CPU-time, address-space
and file-size limits of :mod:`omnicoder.sfb.sandbox`. A candidate passes when the test script exits 0 and prints
its completion marker. ``pass_at_k`` draws k candidates and passes when any one does, which is how the reference's
SFB code factor, its arbiter and its benchmark sweep call it.

CLI: ``python -m omnicoder.eval.code_eval --tasks tasks.jsonl --samples 5`` with rows
``{"candidates": [src, ...], "tests": src}``; prints ``pass@k: passed/total = rate``.
"""
from __future__ import annotations

import argparse
import json
import os
import random
import signal
import sys
import tempfile

from ..sfb.sandbox import _run

_DONE = "__omnicoder_code_eval_done__"


def run_python(code: str, tests: str, timeout: float = 2, mem_bytes: int = 4 << 30) -> tuple[bool, str, str]:
    """Run ``tests`` against ``code``; returns (passed, stdout, stderr). A timeout returns stdout "TIMEOUT"."""
    with tempfile.TemporaryDirectory() as td:
        with open(os.path.join(td, "sol.py"), "w", encoding="utf-8") as f:
            f.write(code)
        with open(os.path.join(td, "test.py"), "w", encoding="utf-8") as f:
            f.write(f"{tests}\nprint({_DONE!r})\n")
        # -E -s (not -I): the script's folder stays on sys.path so the tests can import sol
        r = _run([sys.executable, "-E", "-s", "test.py"], td, int(max(1, round(timeout))), mem_bytes)
    # the wall-clock limit (no return code) or the CPU-time limit (SIGXCPU, then SIGKILL) ended it
    if r.returncode is None or r.returncode in (-signal.SIGXCPU, -signal.SIGKILL):
        return False, "TIMEOUT", ""
    out = r.stdout.replace(_DONE + "\n", "")
    return bool(r.ok and _DONE in r.stdout), out, r.stderr


def pass_at_k(solutions: list[str], tests: str, k: int = 5, timeout: float = 2, seed: int | None = None) -> bool:
    """True when any of k candidates drawn without replacement passes ``tests``."""
    if not solutions:
        return False
    rng = random.Random(seed)
    for s in rng.sample(list(solutions), min(k, len(solutions))):
        if run_python(s, tests, timeout=timeout)[0]:
            return True
    return False


def evaluate_tasks(rows: list[dict], k: int = 5, timeout: float = 2, seed: int | None = 0) -> dict:
    """rows: {"candidates": [...], "tests": str}; returns passed / total / rate."""
    passed = sum(int(pass_at_k(r["candidates"], r["tests"], k=k, timeout=timeout, seed=seed)) for r in rows)
    return {"passed": passed, "total": len(rows), "rate": passed / max(1, len(rows)), "k": k}


def main(argv: list[str] | None = None) -> dict:
    ap = argparse.ArgumentParser(description="pass@k of candidate programs against per-task tests")
    ap.add_argument("--tasks", required=True, help="JSONL rows {candidates: [...], tests: str}")
    ap.add_argument("--samples", type=int, default=5)
    ap.add_argument("--timeout", type=float, default=2)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    with open(args.tasks, encoding="utf-8") as f:
        rows = [json.loads(line) for line in f if line.strip()]
    res = evaluate_tasks(rows, k=args.samples, timeout=args.timeout, seed=args.seed)
    print(f"pass@{args.samples}: {res['passed']}/{res['total']} = {res['rate']:.3f}")
    return res


if __name__ == "__main__":
    main()
