"""Structured factor blending pipeline (factorisation, belief propagation, SPN cache, fusion,
arbiter) and the model-driven tree / graph searches, on CPU."""
import json

import pytest
import torch

from omnicoder.sfb import (BeliefPropagation, CrossBiasFusion, ProofMarginArbiter, ProofMarginInputs, SPNCompiler,
                           factorize_prompt, sfb_bias)


def test_factorize_prompt_factors_and_priors():
    r = factorize_prompt('1. Implement a python function "fib" that must run in at most 10 steps\n'
                         "2. compute the sum of Fibonacci numbers")
    names = {f.name for f in r.factors}
    assert {"subgoals", "entities", "constraints"} <= names
    goals = next(f for f in r.factors if f.name == "subgoals").meta["goals"]
    assert [g["kind"] for g in goals] == ["code", "math"]
    ents = next(f for f in r.factors if f.name == "entities").meta["entities"]
    assert "fib" in ents and "10" in ents and "Fibonacci" in ents
    assert r.goal_priors["code"] > 0.5 and r.goal_priors["math"] > 0.4


def test_belief_propagation_coupling_and_cache():
    r = factorize_prompt("implement python code to solve the equation")
    bp = BeliefPropagation()
    marg = bp.marginals(r)
    assert set(marg) >= {"code", "math"} and all(0 < v < 1 for v in marg.values())
    # the code-math coupling lifts both marginals above their priors
    assert marg["code"] > r.goal_priors["code"] and marg["math"] > r.goal_priors["math"]
    spn = SPNCompiler()
    net = spn.maybe_compile(r)
    assert net is spn.maybe_compile(r) and spn.lookup(r) is None
    msgs = bp.run(r)
    spn.register(r, msgs)
    assert spn.lookup(r) is msgs and all({"prefer_strings", "score"} <= set(m) for m in msgs)


def test_cross_bias_and_pipeline():
    enc = lambda t: [ord(c) % 100 for c in t]
    msgs = [{"prefer_strings": ["ab"], "score": 1.0}, {"prefer_strings": ["zz"], "score": 0.0}]
    b = CrossBiasFusion(enc).bias(msgs, 100)
    assert b[ord("a") % 100] > 0 and b[ord("z") % 100] < 0
    full = sfb_bias("compute xyz", enc, 100)
    assert full.shape == (100,) and full[ord("x") % 100] > full[ord("q") % 100]
    with pytest.raises(RuntimeError):
        CrossBiasFusion().bias(msgs, 100)


def test_proof_margin_arbiter(tmp_path):
    arb = ProofMarginArbiter(threshold=1.0, log_path=str(tmp_path / "log.jsonl"))
    good = ProofMarginInputs(llm_confidence=0.9, sum_log_factors=0.2, verifier_score=0.8, retrieval_hits=2)
    bad = ProofMarginInputs(llm_confidence=0.1, sum_log_factors=-2.0, verifier_score=0.1)
    assert arb.compute_margin(good) == pytest.approx(1.9) and arb.accept(good) and not arb.accept(bad)
    sug = arb.suggestions(bad)
    assert sug["request_retrieval"] and sug["request_resolve"] and sug["bump_scmoe_topk"]
    assert arb.suggestions(good) == {}
    for x, y in [(good, True), (bad, False)] * 10:
        arb.log_decision(x, y)
    w = ProofMarginArbiter.fit_weights_from_log(str(tmp_path / "log.jsonl"))
    assert set(w) == {"w_text", "w_code", "w_img", "w_audio", "w_video"} and w["w_text"] > 1.0


def test_lm_tree_and_graph_search():
    from omnicoder.config import AttentionConfig, ModelConfig
    from omnicoder.models.lm import build_model
    from omnicoder.reasoning.lm_search import LMAdaptiveGraph, LMToTMCTS, ToTConfig
    from omnicoder.training.tokenizer import get_tokenizer
    cfg = ModelConfig(name="s", vocab_size=300, d_model=32, n_layers=1, n_heads=2, ffn_dim=64, max_seq_len=64,
                      attn=AttentionConfig(kind="mha"))
    m = build_model(cfg, device="cpu", seed=0).eval()
    tok = get_tokenizer(cfg.vocab_size)
    best, st = LMToTMCTS(m, tok, ToTConfig(branch=2, max_depth=3, iterations=12, rollout=2)).search("ab")
    assert 1 <= len(best) <= 3 and isinstance(st["text"], str)
    out = LMAdaptiveGraph(m, k=2, thought_len=2, rounds=2, beam=1).step(torch.tensor([[5, 6, 7]]))
    assert out.shape[1] == 3 + 4 and torch.equal(out[0, :3], torch.tensor([5, 6, 7]))


def test_omega_scm_goals_margins_planner():
    from omnicoder.reasoning import omega as om
    # SCM: X -> Y = 2 X (+ noise), Y -> Z = Y + 1
    scm = om.SCM()
    scm.add_variable("X", 1.0)
    scm.add_mechanism("Y", lambda v: 2 * v["X"], parents=["X"])
    scm.add_mechanism("Z", lambda v: v["Y"] + 1, parents=["Y"])
    assert scm.order() == ["X", "Y", "Z"]
    assert scm.forward()["Z"] == 3.0
    assert scm.do({"Y": 10})["Z"] == 11 and scm.do({"X": 2.0})["Z"] == 5.0
    # observed Y = 2.5 at X = 1 -> noise 0.5; had X been 2, Y = 4.5, Z = 5.5
    cf = scm.counterfactual({"X": 1.0, "Y": 2.5, "Z": 3.5}, {"X": 2.0})
    assert abs(cf["Y"] - 4.5) < 1e-9 and abs(cf["Z"] - 5.5) < 1e-9
    assert om.abductive_score(scm, {"Z": 3.0, "Y": 2.0}) == 1.0
    assert om.value_of_information({"a": 0.2, "b": 0.9}, 1) == [("b", 0.9)]
    q = om.build_minimal_scm_for_query("why does the code fail the test")
    assert q.variables["G"].value == 0.7 and q.variables["P"].value == 0.7 and q.forward()["A"] > 0.6
    cyc = om.SCM()
    cyc.add_variable("a", parents=["b"])
    cyc.add_variable("b", parents=["a"])
    with pytest.raises(ValueError):
        cyc.order()
    # goals
    b = om.infer_goals("please fix this crash, error in the traceback, then verify with a test")
    assert b.top() == "debug" and "must-verify" in b.constraints
    assert abs(sum(h.posterior for h in om.infer_goals("x", k=10).hypotheses) - 1.0) < 1e-6
    mem = om.infer_goals("hello", memory={"summarize": 50})
    assert mem.top() == "summarize"
    # margins and certificate
    assert om.text_margin("the cat sat", "a cat sat down") == 2 / 3
    assert om.code_margin(passed=3, total=4) == 0.75
    c = om.pack_certificate("42", b, {"text": 1.0, "image_z": 0.0})
    assert abs(c.margin - 0.75) < 1e-9 and '"answer": "42"' in c.to_json()
    # planner: reach 3 from 0 with +1 / +2 steps; value = closeness
    act, v = om.plan_search(0, lambda s: [1, 2] if s < 3 else [], lambda s, a: s + a,
                            lambda s: 1.0 if s == 3 else 0.0, budget=64, max_depth=3)
    assert act in (1, 2) and v > 0.4
    tb = om.TemplateBank()
    tb.add([1, 0], "a")
    tb.add([0, 1], "b")
    assert tb.query([0.9, 0.1])[0][1] == "a"
    st = om.SymbolicState()
    st.apply("fact: x > 0\ngoal: prove y\nfact: z\nretract: z\ndone: nothing")
    assert st.render_context() == "FACT x > 0\nGOAL prove y"
    om.register_kv_hint((1, 2, 3), "kv123")
    assert om.get_kv_hint((1, 2, 3, 4)) == ((1, 2, 3), "kv123") and om.get_kv_hint((9,)) is None
    assert om.select_branch([(-1.0, 0.2, 7), (-0.5, 0.1, 8)]) == 8
    assert "shortest path" in om.algorithm_hints("find the shortest path in a graph")


def test_code_sandboxes():
    from omnicoder.sfb.sandbox import CppSandbox, HTTPSandbox, PythonSandbox
    py = PythonSandbox()
    ok = py.run("def add(a, b):\n    return a + b", "assert add(2, 3) == 5\nprint('sum', add(1, 1))")
    assert ok.ok and "sum 2" in ok.stdout
    bad = py.run("def add(a, b):\n    return a - b", "assert add(2, 3) == 5")
    assert not bad.ok and "AssertionError" in bad.stderr
    early = py.run("import sys", "sys.exit(0)")
    assert not early.ok                                   # exited before the end marker
    slow = py.run("import time", "time.sleep(30)", timeout=1)
    assert not slow.ok and slow.stderr == "timeout"
    import shutil
    if shutil.which("g++"):
        c = CppSandbox().run("#include <cassert>\nint sq(int x){return x*x;}", "assert(sq(3)==9);")
        assert c.ok
        assert not CppSandbox().run("int f(){return 1;}", "return f();").ok
    assert not HTTPSandbox("http://127.0.0.1:9/none").run("x=1", timeout=1).ok


def test_multi_solution_variants(tmp_path):
    import json

    from omnicoder.training.multi_solution import canonical, code_variants, main, math_variants, rename_locals
    src = ("import math\nTOTAL = 3\n\ndef f(n, scale=2):\n    acc = 0\n    for i in range(n):\n"
           "        acc += i * scale\n    try:\n        q = 1 / n\n    except ZeroDivisionError as e:\n"
           "        q = 0\n    sq = [i * i for i in range(n)]\n    g = lambda z: z + acc\n"
           "    s = 'i q acc'\n    return acc + TOTAL + q + sum(sq) + g(1) + math.floor(1.5) + len(s)\n")
    alt = rename_locals(src)
    assert "for v" in alt and "'i q acc'" in alt and "except ZeroDivisionError as e" in alt
    ns1, ns2 = {}, {}
    exec(src, ns1)
    exec(alt, ns2)
    assert all(ns1["f"](n) == ns2["f"](n) for n in (0, 1, 5))
    assert canonical("x = ( 1+2 )\n") == "x = 1 + 2"
    tests = "from solution import f\n\ndef test_f():\n    assert f(3) == 9\n"
    vs = code_variants("def f(n):\n    t = n*n  # square\n    return t\n", tests)
    assert {v["variant"] for v in vs} == {"rename_locals", "canonical"} and all(v["verified"] for v in vs)
    mv = {v["variant"]: v for v in math_variants("x**2 - 5*x + 6 = 0")}
    assert mv["solved"]["solution"] == "x = 2, x = 3" and mv["factored"]["verified"]
    inp = tmp_path / "m.jsonl"
    inp.write_text(json.dumps({"question": "solve", "answer": "2*y + 4 = 10"}) + "\n")
    out = tmp_path / "o.jsonl"
    assert main(["--input", str(inp), "--domain", "math", "--out", str(out)]) == 0
    rows = [json.loads(ln) for ln in out.read_text().splitlines()]
    assert {r["alt_solution"] for r in rows} >= {"y = 3", "2*y - 6 = 0"}
