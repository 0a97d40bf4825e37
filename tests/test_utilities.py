"""Operational tools (omnicoder.tools.utilities): each subcommand through its CLI entry on CPU."""
import json
import os

import torch

from omnicoder.tools import utilities as U


def _cli(argv) -> int:
    return U.main(argv)


def test_presets_export_and_threshold(tmp_path):
    out = tmp_path / "p.json"
    assert _cli(["presets-export", "--out", str(out), "--names", "tiny_moe", "mobile_2gb"]) == 0
    data = json.loads(out.read_text())
    assert set(data) == {"tiny_moe", "mobile_2gb"} and data["mobile_2gb"]["n_layers"] == 8
    m = tmp_path / "m.json"
    assert _cli(["metrics-canary", "--preset", "tiny_moe", "--prompt_len", "4", "--new_tokens", "4", "--out", str(m),
                 "--device", "cpu"]) == 0
    tps = json.loads(m.read_text())["tokens"]["tokens_per_second"]
    assert tps > 0
    assert _cli(["threshold-check", "--metrics_json", str(m), "--min_tps", str(tps / 2)]) == 0
    assert _cli(["threshold-check", "--metrics_json", str(m), "--min_tps", str(tps * 1e6)]) == 2
    assert _cli(["threshold-check", "--metrics_json", str(tmp_path / "absent.json")]) == 3


def test_package_validate_and_budgets(tmp_path):
    from omnicoder.config import get_preset
    from omnicoder.export.onnx_export import write_sidecars
    from omnicoder.models.lm import build_model
    from omnicoder.tools.export_to_phone import export_for_phone
    model = build_model(get_preset("tiny_moe"), dtype=torch.float32).eval()
    root = tmp_path / "phone"
    export_for_phone(model, str(root), onnx=False, gguf=True, runtimes=False)
    assert _cli(["weights-validate", "--root", str(root)]) == 0
    # a corrupted int4 file is caught by its checksum, a missing required file by name
    f = next(p for p in (root / "int4").iterdir() if p.name != "manifest.json")
    b = bytearray(f.read_bytes())
    b[-1] ^= 0xFF
    f.write_bytes(bytes(b))
    r = U.validate_package(str(root), ("phone_manifest.json", "decode_step.onnx"))
    assert not r["ok"] and any("checksum" in p for p in r["problems"]) and "missing: decode_step.onnx" in r["problems"]

    # resident budget: weights (int4 package) + KV + activations; int8 KV is smaller than bf16
    out = tmp_path / "mb.json"
    assert _cli(["mobile-budget", "--release_root", str(root), "--target_ctx", "256", "--kvq", "int8",
                 "--budget_gb", "4", "--out", str(out)]) == 0
    mb = json.loads(out.read_text())
    assert mb["pass"] and mb["weights_bytes"] > 0 and mb["kv_bytes"] > 0
    cfg = model.cfg
    assert U.kv_bytes_at(cfg, 1024, "int8") < U.kv_bytes_at(cfg, 1024, "bf16")
    assert U.kv_bytes_at(cfg, 1024, "nf4") < U.kv_bytes_at(cfg, 1024, "u8")
    assert _cli(["mobile-budget", "--release_root", str(root), "--target_ctx", "256", "--budget_gb", "1e-6",
                 "--out", str(out)]) == 2

    # KV budget from the exporter's own sidecars (paging + u8 quantisation)
    onnx_path = str(tmp_path / "ds.onnx")
    side = write_sidecars(model, onnx_path, max_len=512, kv_page_len=128, kvq="u8", kvq_group=64)
    paging, kvq = side
    full = U.kv_bytes_from_sidecar(json.load(open(paging)))
    quant = U.kv_bytes_from_sidecar(json.load(open(paging)), json.load(open(kvq)))
    assert quant < full
    assert full == U.kv_bytes_at(cfg, 512, "bf16") + cfg.n_layers * 2 * (cfg.attn.kind == "mla")
    assert _cli(["kv-budget", "--sidecar", paging, "--max_kv_mb", "1024", "--out", str(tmp_path / "k.json")]) == 0
    assert _cli(["kv-budget", "--sidecar", paging, "--max_kv_mb", "1e-6", "--out", str(tmp_path / "k.json")]) == 2
    # the reference's sidecar form: layers * heads * dl * page_len * 2 + spill
    assert U.kv_bytes_from_sidecar({"page_len": 4, "n_layers": 2, "heads": 3, "dl": 5, "spill_bytes": 7}) == \
        2 * 3 * 5 * 4 * 2 + 7


def test_kv_calibrate_static_u8(tmp_path):
    from omnicoder.config import get_preset
    from omnicoder.models.lm import build_model
    model = build_model(get_preset("tiny_moe"), dtype=torch.float32).eval()
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(1, model.cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 9)]
    r = U.kv_calibrate(model, prompts, group=32)
    assert len(r["layers"]) == model.cfg.n_layers
    p = r["layers"][0]["k"]
    assert (p["max"] >= p["min"]).all() and (p["u8_zero"] >= 0).all() and (p["u8_zero"] <= 255).all()
    # 8-bit static parameters from the data itself reproduce it to well under 1 %
    assert max(r["u8_rel_err"]) < 1e-2
    out = tmp_path / "kvq.json"
    assert _cli(["kv-calibrate", "--preset", "tiny_moe", "--max_tokens", "16", "--scheme", "nf4", "--out",
                 str(out)]) == 0
    d = json.loads(out.read_text())
    assert d["scheme"] == "nf4" and len(d["params"]) == model.cfg.n_layers and "absmax" in d["params"][0]["k"]


def test_pq_build_save_load(tmp_path):
    from omnicoder.retrieval.pq import PQRetriever
    docs = tmp_path / "docs"
    docs.mkdir()
    topics = ["cuda kernels tensor cores shared memory", "python lists dictionaries loops",
              "sql joins indexes queries", "rust borrow checker lifetimes"]
    for i in range(12):
        (docs / f"d{i}.txt").write_text(f"{topics[i % 4]} note {i}")
    out = tmp_path / "idx"
    assert _cli(["pq-build", str(docs), str(out), "--m", "4", "--ks", "4", "--dim", "16"]) == 0
    prof = json.loads((out / "budget_profile.json").read_text())
    assert prof["docs"] == 12 and prof["codes_bytes"] == 12 * 4
    pq = PQRetriever.load(str(out))
    hit = pq.search("tensor cores kernels", k=3)
    assert any("cuda" in d for _, _, d in hit)
    assert _cli(["pq-build", str(tmp_path / "empty"), str(out)]) == 3


def test_router_ablate_and_env_audit(tmp_path, monkeypatch):
    out = tmp_path / "r.json"
    assert _cli(["router-ablate", "--routers", "topk", "llm", "hierarchical", "--n_layers", "1", "--d_model", "64",
                 "--n_experts", "4", "--vocab_size", "256", "--max_new_tokens", "2", "--out_json", str(out),
                 "--device", "cpu"]) == 0
    r = json.loads(out.read_text())
    assert set(r["tokens_per_second"]) == {"topk", "llm", "hierarchical"} and r["speedup_x"]["topk"] == 1.0

    src = tmp_path / "src"
    src.mkdir()
    (src / "m.py").write_text('import os\na = os.environ.get("OMNICODER_A", "1")\nb = os.getenv("OMNICODER_B")\n')
    ex = tmp_path / "env.example"
    ex.write_text("OMNICODER_A=1\n# OMNICODER_OLD=0\n")
    monkeypatch.setenv("OMNICODER_STRAY", "x")
    r = U.env_audit(str(src), str(ex))
    assert r["used_not_documented"] == ["OMNICODER_B"] and r["documented_not_used"] == ["OMNICODER_OLD"]
    assert "OMNICODER_STRAY" in r["unknown_set"]
    args = ["env-audit", "--root", str(src), "--env_example", str(ex), "--out_json", str(tmp_path / "e.json"),
            "--out_index", str(tmp_path / "e.md")]
    assert _cli(args + ["--fail_on_drift"]) == 1
    assert _cli(args + ["--sync_example"]) == 0 and "OMNICODER_B" in ex.read_text()
    assert "OMNICODER_A" in (tmp_path / "e.md").read_text()


def test_gen_predictions(tmp_path):
    rows = []
    for i in range(2):
        p = tmp_path / f"img{i}.pt"
        torch.save(torch.rand(3, 32, 32) * 2 - 1, p)
        rows.append({"image": str(p), "question": f"what is {i}?", "answer": str(i)})
    inp = tmp_path / "vqa.jsonl"
    inp.write_text("\n".join(json.dumps(r) for r in rows) + "\n")
    out = tmp_path / "pred.jsonl"
    assert _cli(["gen-predictions", "--task", "vqa", "--input", str(inp), "--out", str(out), "--image_size", "32",
                 "--max_new_tokens", "2", "--device", "cpu"]) == 0
    pred = [json.loads(ln) for ln in out.read_text().splitlines()]
    assert len(pred) == 2 and all("prediction" in p and p["answer"] == str(i) for i, p in enumerate(pred))
    assert os.path.getsize(out) > 0


def test_teacher_verify_agreement(tmp_path):
    from omnicoder.config import get_preset
    from omnicoder.eval import teacher_verify as TV
    from omnicoder.models.lm import build_model
    assert TV.partial_ratio("abc", "xxABCxx") == 1.0 and TV.partial_ratio("", "a") == 0.0
    assert 0.8 < TV.partial_ratio("hello world", "say hello wrld") < 1.0
    assert TV.partial_ratio("abc", "xyz") == 0.0
    model = build_model(get_preset("tiny_moe"), dtype=torch.float32, seed=0)
    ck = tmp_path / "s.pt"
    torch.save({"model": model.export_state_dict(), "config": model.cfg.to_dict()}, ck)
    data = tmp_path / "d.jsonl"
    data.write_text("\n".join(json.dumps(r) for r in [{"prompt": "def add(a, b):", "target": "return a + b"},
                                                      {"question": "2 + 2 =", "answer": "4"}]) + "\n")
    out = tmp_path / "tv.json"
    assert TV.main(["--data", str(data), "--student_ckpt", str(ck), "--teachers", str(ck), "--max_new_tokens", "4",
                    "--out", str(out), "--device", "cpu"]) == 0
    r = json.loads(out.read_text())
    # the same checkpoint as teacher decodes the same greedy tokens: full agreement
    assert r["samples"] == 2 and r["teachers"][str(ck)]["agreement"] == 1.0
    assert 0.0 <= r["overall"]["student_vs_target"] <= 1.0


def test_latent_refine(tmp_path):
    import numpy as np
    from omnicoder.multimodal.video import LatentRefiner
    x = np.random.default_rng(0).standard_normal((2, 5, 16)).astype(np.float32)
    inp, out = tmp_path / "z.npy", tmp_path / "r.npy"
    np.save(inp, x)
    # no checkpoint: the latents pass through unchanged
    assert _cli(["latent-refine", "--latents", str(inp), "--out_latents", str(out)]) == 0
    assert np.allclose(np.load(out), x)
    torch.manual_seed(0)
    ref = LatentRefiner(16, temporal=True)
    torch.save({"refiner": ref.state_dict()}, tmp_path / "ref.pt")
    assert _cli(["latent-refine", "--latents", str(inp), "--out_latents", str(out), "--ckpt",
                 str(tmp_path / "ref.pt"), "--temporal"]) == 0
    with torch.no_grad():
        want = ref(torch.from_numpy(x)).numpy()
    assert np.allclose(np.load(out), want, atol=1e-6)


def test_cycle_consistency(tmp_path):
    from omnicoder.eval.cycle_consistency import cycle_records, main
    d = tmp_path / "gen"
    d.mkdir()
    torch.save(torch.rand(3, 32, 32) * 2 - 1, d / "a.pt")
    torch.save(torch.rand(3, 32, 32) * 2 - 1, d / "b.pt")
    (d / "speech.wav").write_bytes(b"RIFF")
    (d / "notes.md").write_text("ignored")
    (d / "prompts.jsonl").write_text(json.dumps({"file": "a.pt", "prompt": "a red square"}) + "\n")
    (d / "b.txt").write_text("a blue circle")
    (d / "speech.txt").write_text("hello world")
    caps = {"a.pt": "a red square on white", "b.pt": "a green triangle"}
    recs, summary = cycle_records(str(d), caption=lambda p: caps[os.path.basename(p)],
                                  transcribe=lambda p: "hello world")
    by = {os.path.basename(r["file"]): r for r in recs}
    assert set(by) == {"a.pt", "b.pt", "speech.wav"}
    assert by["a.pt"]["agreement"] == 1.0 and by["b.pt"]["agreement"] < 0.7
    assert by["speech.wav"]["agreement"] == 1.0 and summary["audio"]["files"] == 1
    assert summary["image"]["mean_agreement"] == (1.0 + by["b.pt"]["agreement"]) / 2
    out = tmp_path / "cc.jsonl"
    assert main(["--media_dir", str(d), "--image_size", "32", "--out", str(out)]) == 0
    assert len(out.read_text().splitlines()) == 3


def test_act_calibrate_and_validate(tmp_path):
    from omnicoder.models.compat import OmniTransformer
    out = tmp_path / "act.json"
    assert _cli(["act-calibrate", "--preset", "tiny_moe", "--max_tokens", "8", "--decode_steps", "2", "--out",
                 str(out)]) == 0
    d = json.loads(out.read_text())
    from omnicoder.config import get_preset
    cfg = get_preset("tiny_moe")
    # every block's two norms (and the final norm) are GEMM inputs of d_model channels
    assert len(d["modules"]) >= 2 * cfg.n_layers and all(len(v["absmax"]) == cfg.d_model
                                                         for k, v in d["modules"].items() if "norm" in k)
    assert _cli(["act-validate", "--policy", str(out)]) == 0
    d["modules"][next(iter(d["modules"]))]["int8_scale"][0] = float("nan")
    (tmp_path / "bad.json").write_text(json.dumps(d))
    assert _cli(["act-validate", "--policy", str(tmp_path / "bad.json")]) == 2
    # the reference-layout model: Linear / LayerNorm outputs through its own decode path
    torch.manual_seed(0)
    m = OmniTransformer(vocab_size=128, n_layers=1, d_model=32, n_heads=4, mlp_dim=64, n_experts=2, top_k=1,
                        kv_latent_dim=16, use_hrm=False).eval()
    st = U.collect_activation_scales(m, [[1, 2, 3]], decode_steps=2)
    assert any(k.endswith("lm_head") for k in st) and all(torch.isfinite(v).all() for v in st.values())
    # policy sidecar in the reference's form
    pol = tmp_path / "p.act_quant.json"
    pol.write_text(json.dumps({"conf_floor": 0.4, "min_bits": 8, "max_bits": 4,
                               "thresholds": {"layers": {"1": {"conf_floor": 0.5}, "0": {}}}}))
    r = U.act_validate(json.loads(pol.read_text()))
    assert r["global"] == {"conf_floor": 0.4, "min_bits": 8, "max_bits": 4} and r["per_layer_conf_floor"] == [0.4, 0.5]


def test_kv_dump_autoencoder_retention(tmp_path):
    d = tmp_path / "dump"
    assert _cli(["kv-dump", "--preset", "tiny_moe", "--max_tokens", "24", "--out_dir", str(d)]) == 0
    files = sorted(d.glob("kv_*.pt"))
    from omnicoder.config import get_preset
    cfg = get_preset("tiny_moe")
    e = torch.load(files[0], weights_only=True)
    assert len(files) == 4 and len(e) == cfg.n_layers and e[0]["k"].shape[0] <= 24
    rows = U._kv_rows(str(d))
    dim = rows.shape[1]
    # the closed-form (PCA) autoencoder at full rank reproduces the rows; at lower rank it beats SGD
    _, err_full = U.train_kv_autoencoder(rows, dim, "pca")
    assert err_full < 1e-4
    _, err_pca = U.train_kv_autoencoder(rows, 8, "pca")
    _, err_sgd = U.train_kv_autoencoder(rows, 8, "sgd", steps=50)
    assert err_pca <= err_sgd + 1e-6
    side = tmp_path / "side.json"
    assert _cli(["kv-autoencoder", "--kv_dir", str(d), "--latent", "8", "--out_pt", str(tmp_path / "ae.pt"),
                 "--out_json", str(side)]) == 0
    assert json.loads(side.read_text())["kv_autoencoder"]["latent"] == 8
    assert _cli(["kv-autoencoder", "--kv_dir", str(tmp_path / "none")]) == 3
    ret = tmp_path / "r.json"
    assert _cli(["kv-retention", "--out", str(ret), "--window_size", "1024"]) == 0
    assert json.loads(ret.read_text()) == {"compressive_slots": 4, "window_size": 1024, "schema": 1}


def test_code_verify(tmp_path):
    from omnicoder.sfb.sandbox import verify_with_tests
    tests = "from solution import add\n\ndef test_one():\n    assert add(1, 2) == 3\n\ndef test_two():\n    assert add(2, 2) == 4\n"
    r = verify_with_tests("def add(a, b):\n    return a + b\n", tests)
    assert r.ok and (r.passed, r.failed, r.errors) == (2, 0, 0)
    r = verify_with_tests("def add(a, b):\n    return a - b\n", tests)
    assert not r.ok and r.failed == 2
    r = verify_with_tests("def add(:\n", tests)               # a syntax error is a collection error
    assert not r.ok and r.errors >= 1 and r.passed == 0
    t = tmp_path / "tests_add.py"
    t.write_text(tests)
    out = tmp_path / "v.json"
    assert _cli(["code-verify", "--code_text", "def add(a, b):\n    return a + b\n", "--tests_file", str(t),
                 "--out_json", str(out)]) == 0
    assert json.loads(out.read_text())["passed"] == 2
    assert _cli(["code-verify", "--code_text", "def add(a, b):\n    return 0\n", "--tests_file", str(t),
                 "--out_json", str(out)]) == 2


def test_auto_tune_draft_len(tmp_path):
    # accepted / proposed of 4-draft rounds back to the per-token alpha
    a = 0.8
    ratio = (U.expected_tokens(a, 4) - 1) / 4
    assert abs(U.alpha_from_ratio(ratio, 4) - a) < 1e-9
    # a report made from alpha 0.8 and a draft step costing 5 % of a target step
    c = 0.05
    rep = {"acceptance": {"acceptance": ratio, "draft_len": 4, "plain_tokens_per_s": 100.0,
                          "speculative_tokens_per_s": 100.0 * U.expected_tokens(a, 4) / (4 * c + 1)}}
    out = U.tune_draft_len(rep)
    assert abs(out["alpha"] - a) < 1e-6 and abs(out["cost_ratio"] - c) < 1e-6
    best = max(range(1, 17), key=lambda k: U.expected_tokens(a, k) / (k * c + 1))
    assert out["best_draft_len"] == best and out["generate_flags"] == f"--speculative_draft_len {best}"
    # a draft that is rarely accepted: no k beats plain decoding
    low = {"acceptance": 0.0001, "draft_len": 4, "plain_tokens_per_s": 100.0, "speculative_tokens_per_s": 30.0}
    assert U.tune_draft_len(low)["best_draft_len"] == 0
    (tmp_path / "acc.json").write_text(json.dumps(rep))
    assert _cli(["auto-tune", "--acceptance_json", str(tmp_path / "acc.json"), "--out", str(tmp_path / "t.json")]) == 0
    assert json.loads((tmp_path / "t.json").read_text())["best_draft_len"] == best


def test_plot_metrics_svg(tmp_path):
    import xml.etree.ElementTree as ET
    bench = tmp_path / "b.json"
    bench.write_text(json.dumps({"tokens": {"tokens_per_second": 120.5, "seconds": 2.0}, "name": "x", "ok": True}))
    out = tmp_path / "b.svg"
    assert _cli(["plot-metrics", "--bench_json", str(bench), "--out_svg", str(out)]) == 0
    root = ET.fromstring(out.read_text())
    rects = [e for e in root.iter() if e.tag.endswith("rect")]
    assert len(rects) == 2                                  # the two numbers; strings and booleans skipped
    log = tmp_path / "l.jsonl"
    log.write_text("\n".join(json.dumps({"step": i, "loss": 5.0 / (i + 1), "lr": 1e-3}) for i in range(10)))
    assert _cli(["plot-metrics", "--log_jsonl", str(log), "--keys", "loss,lr", "--out_svg", str(out)]) == 0
    root = ET.fromstring(out.read_text())
    lines = [e for e in root.iter() if e.tag.endswith("polyline")]
    assert len(lines) == 2 and len(lines[0].get("points").split()) == 10


def test_write_threshold(tmp_path):
    marks = [{"text": f"t{i}", "write": int(i % 4 == 0), "score": (0.9 if i % 4 == 0 else 0.1) + i * 1e-3}
             for i in range(20)]
    r = U.write_threshold(marks)
    assert r["acceptance_rate"] == 0.25 and r["from"] == "scores"
    assert sum(m["score"] >= r["threshold"] for m in marks) == 5 and r["f1"] == 1.0
    assert U.write_threshold([{"write": 1}, {"write": 0}])["threshold"] == 0.5
    f = tmp_path / "m.jsonl"
    f.write_text("\n".join(json.dumps(m) for m in marks))
    out = tmp_path / "thr.json"
    out.write_text(json.dumps({"other": 0.3}))
    assert _cli(["write-threshold", "--marks", str(f), "--preset", "p1", "--out", str(out)]) == 0
    d = json.loads(out.read_text())
    assert d["other"] == 0.3 and abs(d["p1"] - r["threshold"]) < 1e-12


def test_kv_prefetch_sidecar_and_pager(tmp_path):
    from omnicoder.config import get_preset
    from omnicoder.export.onnx_export import write_sidecars
    from omnicoder.inference.runtimes import LRUKVPager, PagingConfig
    from omnicoder.models.lm import build_model
    model = build_model(get_preset("tiny_moe"), dtype=torch.float32).eval()
    paging = write_sidecars(model, str(tmp_path / "ds.onnx"), max_len=512, kv_page_len=128)[0]
    out = tmp_path / "pf.json"
    assert _cli(["kv-prefetch", "--out", str(out), "--keep_pages", "8", "--kv_paging_sidecar", paging]) == 0
    assert json.loads(out.read_text()) == {"keep_pages": 2}           # 4 pages per layer -> at most half
    assert U.kv_prefetch(3, {"total_pages": 100}) == {"keep_pages": 3}
    cfg = PagingConfig.from_sidecars(paging, str(out))
    assert (cfg.page_len, cfg.n_layers, cfg.max_pages_ram) == (128, model.cfg.n_layers, 2 * model.cfg.n_layers)
    assert LRUKVPager(cfg) is not None
