"""One-button build, export, benchmark and smoke run: ``python -m omnicoder.tools.press_play``.

Reference: src/omnicoder/tools/press_play.py:1-400 (environment checks, optional
training through lets-gooooo, decode-step export (+ quantisation), automatic
benchmarks, manifest, native and ONNX inference smoke).  Steps here:

  1. environment: python / torch / CUDA devices / this package's sm_100a extension,
     onnx and onnxruntime availability;
  2. model: a checkpoint, or training within a budget (omnicoder.tools.lets_gooooo),
     or random weights of a preset;
  3. export: the on-device package (omnicoder.tools.export_to_phone: int4 weights,
     GGUF, ONNX decode step when `onnx` is installed);
  4. benchmarks: native decode tokens/s (omnicoder.inference.benchmark) and, through
     the decode-step runner, tokens/s of the exported step (onnxruntime, or the same
     step in PyTorch when onnxruntime is missing);
  5. smoke: a short greedy generation from a prompt;
  6. `press_play_manifest.json` with every result.
"""
from __future__ import annotations

import argparse
import json
import os
import platform
import sys
import time


def env_report() -> dict:
    rep = {"python": sys.version.split()[0], "os": platform.system(), "arch": platform.machine()}
    import torch
    rep.update(torch=torch.__version__, cuda=torch.cuda.is_available(), devices=torch.cuda.device_count())
    if torch.cuda.is_available():
        rep["device_name"] = torch.cuda.get_device_name(0)
    try:
        from ..ops import _ext
        rep["extension"] = _ext.available()
    except Exception as e:  # report, do not stop the run
        rep["extension"] = f"unavailable: {e}"
    for mod in ("onnx", "onnxruntime"):
        try:
            rep[mod] = __import__(mod).__version__
        except ImportError:
            rep[mod] = None
    return rep


def main(argv=None):
    ap = argparse.ArgumentParser(description="one-button build, export, benchmark and smoke run")
    ap.add_argument("--out_root", default="weights/release")
    ap.add_argument("--ckpt", default="")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--train", action="store_true", help="train first (lets-gooooo) within --train_budget_minutes")
    ap.add_argument("--train_budget_minutes", type=float, default=10.0)
    ap.add_argument("--bench_device", default="", help="device of the benchmarks (default: cuda when present)")
    ap.add_argument("--bench_tokens", type=int, default=32)
    ap.add_argument("--prompt", default="def fibonacci(n):")
    ap.add_argument("--no_export", action="store_true")
    a = ap.parse_args(argv)
    import torch
    os.makedirs(a.out_root, exist_ok=True)
    man = {"started": time.strftime("%Y-%m-%dT%H:%M:%S"), "env": env_report(), "steps": {}}
    ckpt = a.ckpt
    if a.train and not ckpt:
        from .lets_gooooo import main as lets_go
        t0 = time.time()
        rc = lets_go(["--budget_minutes", str(a.train_budget_minutes), "--out_dir", os.path.join(a.out_root, "train"),
                      "--preset", a.preset, "--no_package"])
        man["steps"]["train"] = {"rc": rc, "seconds": round(time.time() - t0, 1)}
        cand = os.path.join(a.out_root, "train", "pretrain.pt")
        ckpt = cand if rc == 0 and os.path.exists(cand) else ""
    from ..inference.builders import build_mobile_model_by_name, load_model
    if ckpt:
        model, _ = load_model(ckpt, "cpu", dtype=torch.float32, preset=a.preset)
    else:
        model = build_mobile_model_by_name(a.preset)
    model = model.eval()
    man["steps"]["model"] = {"source": ckpt or f"random {a.preset}",
                             "params": sum(p.numel() for p in model.parameters())}
    if not a.no_export:
        from .export_to_phone import export_for_phone
        t0 = time.time()
        exp = export_for_phone(model, os.path.join(a.out_root, "export"))
        man["steps"]["export"] = {"artifacts": exp["artifacts"], "seconds": round(time.time() - t0, 1)}
    dev = a.bench_device or ("cuda" if torch.cuda.is_available() else "cpu")
    from ..inference.benchmark import bench_tokens_per_second
    from ..inference.runtimes import TorchStepSession, bench_decode
    bm = model.to(dev) if dev == "cpu" else build_mobile_model_by_name(a.preset, device=dev)
    if dev != "cpu" and ckpt:
        bm.load_state_dict(model.state_dict())
    man["steps"]["bench_native"] = {"device": dev, "tokens_per_s": bench_tokens_per_second(
        bm.eval(), seq_len=32, gen_tokens=a.bench_tokens)}
    sess, kind = None, "torch step (the exported graph's function in PyTorch)"
    onnx_path = os.path.join(a.out_root, "export", "decode_step.onnx")
    if os.path.exists(onnx_path) and man["env"].get("onnxruntime"):
        from ..inference.runtimes import open_session
        sess, kind = open_session(onnx_path), "onnxruntime"
    if sess is None:
        sess = TorchStepSession(model, max_len=32 + a.bench_tokens)
    man["steps"]["bench_decode_step"] = {"session": kind, "tokens_per_s": bench_decode(
        sess, model.cfg.vocab_size, prompt_len=16, gen_tokens=a.bench_tokens)}
    from ..inference.generate import generate
    from ..training.tokenizer import get_tokenizer
    tok = get_tokenizer(model.cfg.vocab_size)
    ids = torch.tensor([tok.encode(a.prompt)], device=dev)
    out = generate(bm, ids, 16, temperature=0.0)
    man["steps"]["smoke"] = {"prompt": a.prompt, "text": tok.decode(out[0, ids.shape[1]:].tolist())}
    man["finished"] = time.strftime("%Y-%m-%dT%H:%M:%S")
    with open(os.path.join(a.out_root, "press_play_manifest.json"), "w") as f:
        json.dump(man, f, indent=1, default=str)
    print(json.dumps(man, indent=1, default=str))
    return 0


if __name__ == "__main__":
    sys.exit(main())
