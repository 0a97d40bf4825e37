"""Rewards computed by programs, for the RL loops (reference src/omnicoder/eval/programmatic_rewards.py:1-69).

* ``code_tests_reward``: fraction of ``_assert(cond)`` checks in a test script that hold for a candidate
  program. The candidate is ``sol.py`` beside the script; the script runs in the sandbox child interpreter
  and reports its counts on a marked line, so prints of the candidate cannot be mistaken for them. A crash,
  a timeout or a script with no checks scores 0.
* ``wer_from_texts``: 1 - word error rate, clipped at 0 (word-level Levenshtein distance over the reference's
  word count). The reference calls jiwer when installed; this is the same quantity from
  :func:`omnicoder.eval.media_metrics.word_error_rate`.
* ``mos_proxy_from_text``: the reference's quality proxy for a text response, 0.5 * (share of letters) +
  0.5 * (1 - |characters - 128| / 128), each clipped to [0, 1].
"""
from __future__ import annotations

import os
import sys
import tempfile

from ..sfb.sandbox import _run
from .media_metrics import word_error_rate

_COUNTS = "__omnicoder_reward_counts__"


def code_tests_reward(candidate_py: str, tests_code: str, timeout_s: float = 3, mem_bytes: int = 4 << 30) -> float:
    runner = (
        "_passed = 0\n_total = 0\n"
        "def _assert(cond):\n    global _passed, _total\n    _total += 1\n    _passed += bool(cond)\n\n"
        f"{tests_code}\n\nprint({_COUNTS!r}, _passed, _total)\n"
    )
    with tempfile.TemporaryDirectory() as td:
        with open(os.path.join(td, "sol.py"), "w", encoding="utf-8") as f:
            f.write(candidate_py)
        with open(os.path.join(td, "tests_runner.py"), "w", encoding="utf-8") as f:
            f.write(runner)
        r = _run([sys.executable, "-E", "-s", "tests_runner.py"], td, int(max(1, round(timeout_s))), mem_bytes)
    for line in reversed(r.stdout.splitlines()):
        parts = line.split()
        if len(parts) == 3 and parts[0] == _COUNTS:
            p, t = int(parts[1]), int(parts[2])
            return p / t if t > 0 else 0.0
    return 0.0


def wer_from_texts(reference: str, hypothesis: str) -> float:
    return max(0.0, 1.0 - word_error_rate(reference, hypothesis))


def mos_proxy_from_text(text: str) -> float:
    txt = text.strip()
    n = len(txt)
    if n == 0:
        return 0.0
    letters = sum(ch.isalpha() for ch in txt) / n
    length = min(1.0, max(0.0, 1.0 - abs(n - 128) / 128.0))
    return min(1.0, max(0.0, 0.5 * letters + 0.5 * length))
