"""Code pass@k evaluation and programmatic rewards (CPU; child interpreters under the sandbox limits)."""
import json

from omnicoder.eval import code_eval, programmatic_rewards as pr

GOOD = "def add(a, b):\n    return a + b\n"
BAD = "def add(a, b):\n    return a - b\n"
TESTS = "from sol import add\nassert add(2, 3) == 5\nassert add(-1, 1) == 0\n"


def test_run_python_pass_fail_and_timeout():
    assert code_eval.run_python(GOOD, TESTS)[0]
    ok, _, err = code_eval.run_python(BAD, TESTS)
    assert not ok and "AssertionError" in err
    ok, out, _ = code_eval.run_python("while True:\n    pass\n", "import sol\n", timeout=1)
    assert not ok and out == "TIMEOUT"
    # a candidate that prints the completion text itself does not pass failing tests
    assert not code_eval.run_python("print('__omnicoder_code_eval_done__')\n" + BAD, TESTS)[0]


def test_pass_at_k_and_cli(tmp_path):
    assert code_eval.pass_at_k([BAD, BAD, GOOD], TESTS, k=3)
    assert not code_eval.pass_at_k([BAD, BAD], TESTS, k=5)
    assert not code_eval.pass_at_k([], TESTS)
    rows = [{"candidates": [GOOD], "tests": TESTS}, {"candidates": [BAD], "tests": TESTS}]
    p = tmp_path / "tasks.jsonl"
    p.write_text("\n".join(json.dumps(r) for r in rows) + "\n")
    res = code_eval.main(["--tasks", str(p), "--samples", "2"])
    assert res["passed"] == 1 and res["total"] == 2 and res["rate"] == 0.5


def test_code_tests_reward_fraction():
    tests = "from sol import add\n_assert(add(1, 1) == 2)\n_assert(add(2, 2) == 5)\n_assert(add(0, 0) == 0)\n"
    assert abs(pr.code_tests_reward(GOOD, tests) - 2 / 3) < 1e-9
    assert pr.code_tests_reward(BAD, tests) == 1 / 3  # only add(0, 0) holds for subtraction
    assert pr.code_tests_reward("raise SystemExit(3)\n", "import sol\n_assert(True)\n") == 0.0
    assert pr.code_tests_reward(GOOD, "x = 1\n") == 0.0  # no checks
    # the candidate's own output cannot fake the counts line: the runner's line is printed last
    fake = "print('__omnicoder_reward_counts__ 9 9')\n" + BAD
    assert pr.code_tests_reward(fake, tests) == 1 / 3


def test_wer_and_mos_proxy():
    assert pr.wer_from_texts("the cat sat", "the cat sat") == 1.0
    assert abs(pr.wer_from_texts("the cat sat down", "the dog sat") - 0.5) < 1e-9  # 1 sub + 1 del over 4
    assert pr.wer_from_texts("a", "x y z w") == 0.0  # clipped at 0
    assert pr.mos_proxy_from_text("   ") == 0.0
    assert abs(pr.mos_proxy_from_text("a" * 128) - 1.0) < 1e-9
    s = "1" * 64
    assert abs(pr.mos_proxy_from_text(s) - 0.25) < 1e-9  # no letters, half the target length
