"""Entry points: pretrain (single process, resume, text folder), the expert-parallel
launcher with 2 CPU ranks (gloo), the training orchestrator, generate CLI."""
import json
import os
import subprocess
import sys

import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, timeout=600):
    env = dict(os.environ, PYTHONPATH=ROOT, CUDA_VISIBLE_DEVICES="")
    r = subprocess.run([sys.executable, "-m"] + args, cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=timeout)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    return r.stdout


def test_pretrain_text_folder_and_resume(tmp_path):
    d = tmp_path / "data"
    d.mkdir()
    (d / "a.txt").write_text("the quick brown fox jumps over the lazy dog. " * 40)
    out, st, log = tmp_path / "m.pt", tmp_path / "s.pt", tmp_path / "log.jsonl"
    common = ["--preset", "tiny_moe", "--seq_len", "32", "--batch_size", "2", "--log_interval", "1", "--device", "cpu",
              "--out", str(out), "--state_out", str(st), "--log_file", str(log)]
    _run(["omnicoder.training.pretrain", "--data", str(d), "--steps", "2"] + common)
    assert out.exists() and st.exists()
    ck = torch.load(out, weights_only=False)
    assert ck["step"] == 2 and any(k.endswith(".w1") for k in ck["model"])
    _run(["omnicoder.training.pretrain", "--data", str(d), "--steps", "3", "--resume_ckpt", str(out),
          "--log_expert_load"] + common)
    recs = [json.loads(l) for l in log.read_text().splitlines()]
    assert [r["step"] for r in recs] == [1, 2, 3]          # the resumed run continues at step 3
    assert "expert_load_cv" in recs[-1] and recs[-1]["model_tflops_per_gpu"] > 0


def test_torchrun_ep_two_cpu_ranks(tmp_path):
    out = _run(["omnicoder.tools.torchrun_ep", "--devices", "cpu,cpu", "--script", "omnicoder.training.pretrain", "--",
                "--device", "cpu", "--data", "synthetic", "--preset", "tiny_moe", "--seq_len", "32", "--batch_size", "2",
                "--steps", "2", "--log_interval", "1", "--out", str(tmp_path / "m.pt"), "--state_out",
                str(tmp_path / "s.pt"), "--log_file", str(tmp_path / "l.jsonl")], timeout=900)
    assert "step 2/2" in out
    ck = torch.load(tmp_path / "m.pt", weights_only=False)
    # rank 0 gathered every rank's experts into one consolidated checkpoint
    assert ck["model"]["blocks.0.ffn.w1"].shape[0] == 4
    assert (tmp_path / "s.pt.rank0").exists() and (tmp_path / "s.pt.rank1").exists()


def test_run_training_plan_dry_run():
    out = _run(["omnicoder.tools.run_training", "--dry_run", "--budget_minutes", "1", "--stages", "pretrain,draft,export"])
    assert "omnicoder.training.pretrain" in out and "onnx_export" in out


def test_press_play_export_to_phone_and_lets_go(tmp_path):
    """One-button run (export, benchmarks, smoke, manifest), the phone package, and the budgeted
    training planner (dry run with a given step rate, distill stage included)."""
    out = tmp_path / "rel"
    _run(["omnicoder.tools.press_play", "--out_root", str(out), "--preset", "tiny_moe", "--bench_tokens", "4"])
    man = json.loads((out / "press_play_manifest.json").read_text())
    assert man["steps"]["bench_native"]["tokens_per_s"] > 0 and man["steps"]["bench_decode_step"]["tokens_per_s"] > 0
    assert (out / "export" / "int4" / "manifest.json").exists() and (out / "export" / "model.gguf").exists()
    ph = tmp_path / "phone"
    o = _run(["omnicoder.tools.export_to_phone", "--preset", "tiny_moe", "--out", str(ph), "--no_gguf", "--push"])
    assert "adb push" in o and json.loads((ph / "phone_manifest.json").read_text())["artifacts"]["int4_package"]
    o = _run(["omnicoder.tools.lets_gooooo", "--dry_run", "--steps_per_minute", "30", "--budget_minutes", "2",
              "--out_dir", str(tmp_path / "lg")])
    assert "omnicoder.training.distill" in o and "omnicoder.training.pretrain" in o


def test_draft_train_pipeline(tmp_path):
    """KD of a LoRA draft, checkpoint, acceptance benchmark; greedy speculative decoding with the
    draft reproduces plain decoding (sequences that finish first stop advancing their cache)."""
    o = _run(["omnicoder.training.draft_train", "--steps", "2", "--seq_len", "32", "--batch_size", "2",
              "--device", "cpu", "--student_preset", "tiny_moe", "--lora", "--out_ckpt", str(tmp_path / "d.pt"),
              "--bench_out", str(tmp_path / "b.json")])
    rep = json.loads((tmp_path / "b.json").read_text())
    assert rep["acceptance"]["same_output"] and (tmp_path / "d.pt").exists()


def test_auto_benchmark_sweep(tmp_path):
    """Throughput per KV format, multiple-choice scoring by log-likelihood, perplexity and the
    prediction-file scorers, written to JSON and CSV."""
    mc = tmp_path / "mc.jsonl"
    mc.write_text("\n".join(json.dumps({"question": f"q{i}?", "choices": ["aa", "bb", "cc"], "answer": i % 3})
                            for i in range(6)))
    vqa = tmp_path / "vqa.jsonl"
    vqa.write_text(json.dumps({"prediction": "Cat", "answer": "cat"}) + "\n" +
                   json.dumps({"prediction": "dog", "answer": "cow"}))
    asr = tmp_path / "asr.jsonl"
    asr.write_text(json.dumps({"prediction": "a b c", "reference": "a b d"}))
    txt = tmp_path / "t.txt"
    txt.write_text("hello world " * 200)
    out = tmp_path / "s.json"
    _run(["omnicoder.eval.auto_benchmark", "--device", "cpu", "--seq_len", "16", "--gen_tokens", "4",
          "--kv", "none,u8,nf4", "--mmlu_jsonl", str(mc), "--arc_jsonl", str(mc), "--vqa_jsonl", str(vqa),
          "--asr_jsonl", str(asr), "--text", str(txt), "--out", str(out), "--out_csv", str(tmp_path / "s.csv")])
    r = json.loads(out.read_text())
    assert r["tokens_per_s_kv_none"] > 0 and r["tokens_per_s_kv_nf4"] > 0
    assert r["mmlu"]["n"] == 6 and 0 <= r["mmlu"]["accuracy"] <= 1
    assert r["vqa_exact_match"] == 0.5 and abs(r["asr_wer"] - 1 / 3) < 1e-6 and r["perplexity"] > 1
    assert (tmp_path / "s.csv").exists()


def test_rl_and_vl_task_clis(tmp_path):
    from omnicoder.training import rl, vl_tasks
    assert rl.main(["--steps", "1", "--batch", "1", "--group", "2", "--max_new_tokens", "4", "--device", "cpu",
                    "--out", str(tmp_path / "rl.pt")]) == 0
    assert (tmp_path / "rl.pt").exists()
    assert vl_tasks.main(["--task", "caption", "--steps", "1", "--batch", "2", "--image_size", "32", "--device", "cpu",
                          "--out", str(tmp_path / "vl.pt")]) == 0
    assert (tmp_path / "vl.pt").exists()


def test_run_training_smoke_one_step(tmp_path):
    out = _run(["omnicoder.tools.run_training", "--stages", "vqa,rl", "--out_dir", str(tmp_path),
                "--smoke_one_step", "--device", "cpu"])
    summary = json.loads(out[out.rindex("{\n \"plan\""):])
    assert all(v["steps"] == 1 for v in summary["plan"].values())
    assert {k: v["rc"] for k, v in summary["results"].items()} == {"vqa": 0, "rl": 0}
    # alignment chain: the concept-head stage picks up the pre-alignment checkpoint
    out = _run(["omnicoder.tools.run_training", "--stages", "pre_align,align,audio_recon", "--out_dir",
                str(tmp_path), "--smoke_one_step", "--device", "cpu"])
    summary = json.loads(out[out.rindex("{\n \"plan\""):])
    assert all(v["rc"] == 0 for v in summary["results"].values()), summary
    assert (tmp_path / "pre_align.pt").exists() and (tmp_path / "concept_head.pt").exists()


def test_verifier_distillation(tmp_path):
    """The verifier head learns the teacher's softened distribution: the KL falls; with
    verifier_only nothing but the verifier moves; a teacher with another vocabulary goes
    through the learned aligner."""
    from omnicoder.config import ModelConfig
    from omnicoder.models.lm import build_model
    from omnicoder.training.verifier_distill import VerifierDistiller, main
    cfg = ModelConfig(name="v", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64,
                      verifier_head=True)
    student = build_model(cfg, "cpu", dtype=torch.float32, seed=0)
    tcfg = ModelConfig(name="t", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64)
    teacher = build_model(tcfg, "cpu", dtype=torch.float32, seed=1).eval()
    before = {n: p.detach().clone() for n, p in student.named_parameters()}
    vd = VerifierDistiller(student, lr=3e-3, verifier_only=True)
    ids = torch.randint(0, cfg.vocab_size, (2, 32))
    with torch.no_grad():
        t = teacher(ids, all_logits=True)["logits"]
    losses = [vd.step(ids, t) for _ in range(8)]
    assert losses[-1] < losses[0]
    moved = [n for n, p in student.named_parameters() if not torch.equal(p, before[n])]
    assert moved == ["verifier"]
    vd2 = VerifierDistiller(student, lr=1e-3, teacher_vocab=cfg.vocab_size + 17)
    t2 = torch.randn(2, 32, cfg.vocab_size + 17)
    assert vd2.step(ids, t2) > 0 and vd2.align.weight.grad is not None
    assert main(["--steps", "1", "--seq_len", "16", "--batch_size", "1", "--device", "cpu",
                 "--out", str(tmp_path / "v.pt")]) == 0


def test_code_expert_router_kd_and_balance(tmp_path):
    from omnicoder.config import ModelConfig, MoEConfig
    from omnicoder.models.lm import build_model
    from omnicoder.training.code_expert import RouterTap, code_expert_loss, main, sinkhorn
    p = sinkhorn(torch.randn(64, 8), iters=30)
    assert torch.allclose(p.sum(1), torch.ones(64), atol=1e-4) and torch.allclose(p.sum(0), torch.full((8,), 8.0),
                                                                                     atol=1e-2)
    cfg = ModelConfig(name="ce", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64,
                      moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=64))
    s = build_model(cfg, "cpu", dtype=torch.float32, seed=0)
    t = build_model(cfg, "cpu", dtype=torch.float32, seed=1).eval()
    st, tt = RouterTap(s), RouterTap(t)
    ids, lab = torch.randint(0, 300, (2, 16)), torch.randint(0, 300, (2, 16))
    loss, parts = code_expert_loss(s, t, st, tt, ids, lab)
    assert set(parts) == {"kd", "router_kd", "balance"} and parts["router_kd"] > 0
    loss.backward()
    routers = [m.router for m in st.layers]
    assert all(r.grad is not None and r.grad.abs().sum() > 0 for r in routers)
    # the router KD term vanishes when the student's routers equal the teacher's
    s2 = build_model(cfg, "cpu", dtype=torch.float32, seed=1)
    st2 = RouterTap(s2)
    _, parts2 = code_expert_loss(s2, t, st2, tt, ids, lab, balance=0.0)
    assert parts2["router_kd"] < 1e-6
    assert main(["--steps", "1", "--seq_len", "16", "--batch_size", "1", "--device", "cpu",
                 "--student_preset", "tiny_moe", "--out", str(tmp_path / "c.pt")]) == 0


def test_run_training_probe_sizes_the_plan(tmp_path):
    """The probe runs each stage for 1 and 3 steps and the plan uses the measured rates."""
    from omnicoder.tools.run_training import plan
    out = _run(["omnicoder.tools.run_training", "--stages", "audio_recon,pre_align", "--out_dir", str(tmp_path),
                "--probe_only", "--device", "cpu"])
    pr = json.loads((tmp_path / "train_probe_summary.json").read_text())
    assert set(pr) == {"audio_recon", "pre_align"} and all(v["rc"] == 0 and v["steps_per_minute"] > 0
                                                           for v in pr.values()), out
    p = plan(10.0, {k: v["steps_per_minute"] for k, v in pr.items()}, ["audio_recon", "pre_align"])
    for s in p:
        assert p[s]["steps"] == max(1, int(p[s]["minutes"] * pr[s]["steps_per_minute"]))
    # an unknown stage in the plan takes the mean measured rate
    q = plan(10.0, {"pre_align": 30.0}, ["pre_align", "audio_recon"])
    assert q["audio_recon"]["steps"] == int(q["audio_recon"]["minutes"] * 30.0)
    out = _run(["omnicoder.tools.run_training", "--stages", "pre_align", "--out_dir", str(tmp_path / "r"),
                "--probe_json", str(tmp_path / "train_probe_summary.json"), "--dry_run"])
    assert "omnicoder.training.pre_align" in out


def test_prepare_data_feeds_the_trainers(tmp_path):
    """Generated workspace data runs through the VQA / unified trainers, the code verifier and the
    write-threshold tool; a rerun writes nothing."""
    from omnicoder.sfb.sandbox import verify_with_tests
    from omnicoder.tools.prepare_data import prepare
    from omnicoder.tools.utilities import main as tools_main
    from omnicoder.training import vl_tasks
    root = tmp_path / "data"
    r = prepare(str(root))
    assert len(r["written"]) > 10 and prepare(str(root))["written"] == []
    task = json.loads((root / "code" / "tasks.jsonl").read_text().splitlines()[2])
    assert verify_with_tests(task["target"], task["tests"]).ok
    assert vl_tasks.main(["--task", "vqa", "--jsonl", str(root / "vl" / "vqa.jsonl"), "--image_size", "32",
                          "--steps", "1", "--batch", "2", "--device", "cpu", "--out", str(tmp_path / "v.pt")]) == 0
    assert vl_tasks.main(["--task", "unified", "--jsonl", str(root / "unified.jsonl"), "--image_size", "32",
                          "--steps", "2", "--batch", "2", "--device", "cpu", "--out", str(tmp_path / "u.pt")]) == 0
    assert tools_main(["write-threshold", "--marks", str(root / "marks.jsonl"), "--out",
                       str(tmp_path / "thr.json")]) == 0
