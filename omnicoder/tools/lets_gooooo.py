"""Budgeted end-to-end training run: ``python -m omnicoder.tools.lets_gooooo``.

Reference: src/omnicoder/tools/lets_gooooo.py:1-120 (one command that trains
within a time budget -- pretraining, distillation, draft model -- and exports the
result).  Here it plans the stages of omnicoder.tools.run_training from the
budget (measuring the step rate with a short probe run unless given), runs them
with a time limit each, resumes finished stages on a rerun, and finishes with the
on-device package (omnicoder.tools.export_to_phone).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time


def probe_steps_per_minute(preset: str, seq_len: int, batch: int, steps: int = 3) -> float:
    """Optimiser steps per minute of `preset` on this machine (a few timed steps)."""
    import torch

    from ..config import TrainConfig, get_preset
    from ..models.lm import build_model
    from ..training.engine import Trainer, synthetic_batch
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    cfg = get_preset(preset)
    model = build_model(cfg, device=dev, seed=0)
    tr = Trainer(model, TrainConfig(lr=1e-4, warmup_steps=0, max_steps=steps + 1))
    b = synthetic_batch(batch, seq_len, cfg.vocab_size, seed=0, step=0, device=dev)
    tr.step(*b)
    if dev == "cuda":
        torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        float(tr.step(*b).loss)
    return 60.0 * steps / max(1e-6, time.perf_counter() - t0)


def main(argv=None):
    ap = argparse.ArgumentParser(description="train within a time budget, then package the model")
    ap.add_argument("--budget_minutes", type=float, default=30.0)
    ap.add_argument("--out_dir", default="weights/lets_go")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--draft_preset", default="draft_2l")
    ap.add_argument("--data", default="synthetic")
    ap.add_argument("--seq_len", type=int, default=256)
    ap.add_argument("--batch_size", type=int, default=4)
    ap.add_argument("--steps_per_minute", type=float, default=0.0, help="0: measure with a probe run")
    ap.add_argument("--stages", default="pretrain,distill,draft")
    ap.add_argument("--teacher_hf", default=None)
    ap.add_argument("--devices", default="")
    ap.add_argument("--no_package", action="store_true")
    ap.add_argument("--dry_run", action="store_true")
    a = ap.parse_args(argv)
    spm = a.steps_per_minute or probe_steps_per_minute(a.preset, a.seq_len, a.batch_size)
    from . import run_training
    args = ["--out_dir", a.out_dir, "--data", a.data, "--budget_minutes", str(a.budget_minutes * 0.95),
            "--steps_per_minute", str(spm), "--stages", a.stages, "--preset", a.preset, "--draft_preset",
            a.draft_preset, "--seq_len", str(a.seq_len), "--batch_size", str(a.batch_size)]
    if a.devices:
        args += ["--devices", a.devices]
    if a.teacher_hf:
        args += ["--teacher_hf", a.teacher_hf]
    if a.dry_run:
        args.append("--dry_run")
    rc = run_training.main(args)
    summary = {"steps_per_minute": spm, "train_rc": rc}
    ckpt = os.path.join(a.out_dir, "pretrain.pt")
    if rc == 0 and not a.no_package and not a.dry_run and os.path.exists(ckpt):
        from .export_to_phone import main as export_main
        export_main(["--ckpt", ckpt, "--preset", a.preset, "--out", os.path.join(a.out_dir, "package")])
        summary["package"] = os.path.join(a.out_dir, "package")
    print(json.dumps(summary))
    return rc


if __name__ == "__main__":
    sys.exit(main())
