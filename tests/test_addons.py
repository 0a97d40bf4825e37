"""Utilities and add-ons: perf counters, logging, env registry, metrics, PQ /
graph retrieval, multimodal front ends, reasoning search, belief propagation,
planning."""
import json
import os

import numpy as np
import torch


def test_perf_logger_env(tmp_path):
    from omnicoder.utils import perf
    from omnicoder.utils.env import load_dotenv, registry_markdown, scan_registry
    from omnicoder.utils.logger import get_logger
    perf.reset()
    with perf.timer("x"):
        sum(range(1000))
    perf.add("x", 0.5)
    snap = perf.snapshot()
    assert snap["x"]["count"] == 2 and snap["x"]["total_s"] >= 0.5
    with perf.nvtx("region"):
        pass
    trace = tmp_path / "t.log"
    perf.enable_call_trace(str(trace))
    json.dumps({})
    perf.disable_call_trace()
    assert "call" in trace.read_text()
    get_logger("test").info("hello")
    reg = scan_registry()
    assert any(k.startswith("OMNICODER_") for k in reg) and "|" in registry_markdown(reg)
    (tmp_path / ".env").write_text("OMNI_TEST_X=1\n# c\n")
    assert load_dotenv(str(tmp_path / ".env")) == {"OMNI_TEST_X": "1"}
    os.environ.pop("OMNI_TEST_X")


def test_metrics():
    from omnicoder.eval import pass_at_k, perplexity
    from omnicoder.config import ModelConfig, AttentionConfig
    from omnicoder.models.lm import build_model
    assert pass_at_k(10, 10, 1) == 1.0 and pass_at_k(10, 0, 1) == 0.0
    assert abs(pass_at_k(10, 3, 1) - 0.3) < 1e-9
    m = build_model(ModelConfig(vocab_size=50, d_model=32, n_layers=1, n_heads=4, ffn_dim=64, max_seq_len=32,
                                attn=AttentionConfig(kind="mha")))
    ppl = perplexity(m, [torch.randint(0, 50, (17,)) for _ in range(2)])
    assert 20 < ppl < 120                      # random init: near the vocabulary size


def test_retrieval():
    from omnicoder.retrieval import GraphRAG, PQRetriever
    docs = ["Paris is the capital of France", "Berlin is the capital of Germany",
            "Python lists support append and pop", "Rust has ownership and borrowing"] * 3
    r = PQRetriever(n_subspaces=4, n_centroids=4, dim=32).fit(docs)
    top = r.search("capital of France Paris", k=3)
    assert any("France" in t[2] for t in top[:2])
    g = GraphRAG().add(["Alice works with Bob", "Bob lives in Paris", "Carol likes Rust"])
    res = g.retrieve("Where does Alice's colleague live?", k=2)
    assert any("Paris" in p for _, p in res)


def test_multimodal():
    from omnicoder.multimodal import MelFrontend, MultimodalComposer, PatchEncoder, VectorQuantizer, VocabSidecar
    from omnicoder.multimodal import map_image_tokens
    lay = VocabSidecar.from_config()
    lay.integrity_checks()
    assert map_image_tokens([0, 5]) == [32000, 32005] and lay.modality_of(32000 + 8192) == "video"
    enc = PatchEncoder(image_size=32, patch=8, dim=32, depth=1, heads=2)
    f = enc(torch.randn(2, 3, 32, 32))
    assert f.shape == (2, 17, 32)
    vq = VectorQuantizer(64, 32)
    q, codes, loss = vq(f)
    assert q.shape == f.shape and int(codes.max()) < 64 and loss >= 0
    mel = MelFrontend(n_mels=20, out_dim=32)(torch.randn(2, 4000))
    comp = MultimodalComposer(32, {"image": 32, "audio": 32})
    seq = comp.fuse_features(torch.randn(2, 5, 32), image=f, audio=mel)
    assert seq.shape == (2, 17 + 2 + mel.shape[1] + 2 + 5, 32)
    ids = comp.fuse_codes(torch.ones(2, 3, dtype=torch.long), image=codes[:, :4])
    assert int(ids[0, 0]) >= 32000


def test_reasoning():
    from omnicoder.reasoning import Action, FactorGraph, TreeOfThoughtsMCTS, plan, self_consistency
    it = iter(["a", "b", "a", "a"])
    assert self_consistency(lambda: next(it), 4) == ("a", 0.75)
    # find the digit string 3-1-4 by search
    target = (3, 1, 4)
    mcts = TreeOfThoughtsMCTS(expand=lambda s: list(range(5)),
                              evaluate=lambda s: sum(a == b for a, b in zip(s, target)) / 3, max_depth=3)
    assert tuple(mcts.search(iterations=400)) == target
    fg = FactorGraph()
    for v in "abc":
        fg.add_variable(v, 2)
    fg.add_factor(("a",), [0.3, 0.7])
    fg.add_factor(("a", "b"), [[0.9, 0.1], [0.2, 0.8]])
    fg.add_factor(("b", "c"), [[0.6, 0.4], [0.3, 0.7]])
    bp, ex = fg.marginals(iters=20), fg.exact_marginals()
    for v in "abc":
        assert np.allclose(bp[v], ex[v], atol=1e-6)
    acts = [Action("pick", frozenset({"hand_empty"}), frozenset({"holding"}), frozenset({"hand_empty"})),
            Action("place", frozenset({"holding"}), frozenset({"placed", "hand_empty"}), frozenset({"holding"}))]
    assert plan({"hand_empty"}, {"placed"}, acts) == ["pick", "place"]
