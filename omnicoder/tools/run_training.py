"""Training orchestrator: ``python -m omnicoder.tools.run_training``.

Runs the stages of a training plan as child processes with a time budget each
(reference src/omnicoder/tools/run_training.py:102-1366: stage planning from a
minute budget, `run_with_timeout`, resume by skipping finished stages, optional
expert-parallel launch).  Stages here: `pretrain` (spec LM), `distill`
(knowledge distillation of the draft-sized student from the pretrained model or
a local Hugging Face teacher), `draft` (small draft model for speculative
decoding), `draft_kd` (draft pipeline: KD with LoRA, export, acceptance),
`code_expert` (code distillation with router KD and balanced routing), `verifier` (verifier-head
distillation), `vl` / `vqa` (vision-language pretraining and VQA
over the fusion composer), `rl`
(GRPO on programmatic rewards), `eval` (evaluation sweep), `export` (ONNX decode
step), `package` (on-device package), `pre_align` / `align` (modality pre-alignment and
the concept head), `flow_recon` / `audio_recon` (latent heads).  `--smoke_one_step` runs one step
of every requested stage (wiring check, the reference's smoke mode); `--probe` first measures each
stage's steps per minute and sizes the plan with the measured rates.  Each stage
writes a marker file when it finishes; a rerun skips finished stages unless
--force is given.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time


def run_with_timeout(cmd: list[str], timeout_s: float, env=None) -> int:
    """Run `cmd`; on timeout terminate its process group and return 124."""
    p = subprocess.Popen(cmd, env=env, start_new_session=True)
    try:
        return p.wait(timeout=timeout_s if timeout_s > 0 else None)
    except subprocess.TimeoutExpired:
        import signal
        os.killpg(p.pid, signal.SIGTERM)
        try:
            p.wait(timeout=30)
        except subprocess.TimeoutExpired:
            os.killpg(p.pid, signal.SIGKILL)
        return 124


def plan(budget_minutes: float, steps_per_minute, stages: list[str]) -> dict:
    """Split the budget by relative shares of the requested stages; `steps_per_minute` is one rate
    for every stage or {stage: rate} (a probe's measurements; missing stages take the mean)."""
    share = {"pretrain": 0.8, "distill": 0.1, "draft": 0.15, "draft_kd": 0.1, "code_expert": 0.1, "verifier": 0.05, "vl": 0.1, "vqa": 0.05, "rl": 0.1,
             "pre_align": 0.05, "align": 0.05, "flow_recon": 0.05, "audio_recon": 0.05, "eval": 0.03, "export": 0.05, "package": 0.03}
    tot = sum(share[s] for s in stages) or 1.0
    if isinstance(steps_per_minute, dict):
        known = [v for v in steps_per_minute.values() if v > 0]
        fallback = sum(known) / len(known) if known else 60.0
        rate = {s: steps_per_minute.get(s, fallback) or fallback for s in stages}
    else:
        rate = {s: steps_per_minute for s in stages}
    return {s: {"minutes": budget_minutes * share[s] / tot,
                "steps": max(1, int(budget_minutes * share[s] / tot * rate[s]))} for s in stages}


def probe(stages: list[str], a, extra_steps: int = 2, probe_dir: str | None = None) -> dict:
    """Measured steps per minute of each stage (the reference's train_probe, tools/train_probe.py:30-218,
    which runs every stage for one step): each stage runs for 1 and for 1 + extra_steps steps in a
    scratch folder, and the rate is extra_steps over the difference of the two wall times, so process
    start-up and model building cancel out."""
    probe_dir = probe_dir or os.path.join(a.out_dir, "probe")
    os.makedirs(probe_dir, exist_ok=True)
    out = {}
    for s in stages:
        times, rc = [], 0
        for n in (1, 1 + extra_steps):
            t0 = time.time()
            rc = run_with_timeout(stage_command(s, a, n, probe_dir), 1800)
            times.append(time.time() - t0)
            if rc != 0:
                break
        if rc != 0:
            out[s] = {"rc": rc, "seconds": [round(t, 2) for t in times]}
            continue
        dt = times[1] - times[0]
        spm = 60.0 * extra_steps / dt if dt > 0.05 * times[1] else 60.0 * (1 + extra_steps) / times[1]
        out[s] = {"rc": 0, "seconds": [round(t, 2) for t in times], "steps_per_minute": round(spm, 2)}
    return out


def stage_command(s: str, a, steps: int, out_dir: str | None = None) -> list[str]:
    """The child-process command of stage `s` for `steps` steps, writing into `out_dir`
    (default: the run's output folder)."""
    out_dir = out_dir or a.out_dir
    a = argparse.Namespace(**{**vars(a), "out_dir": out_dir})
    dev = ["--device", a.device] if a.device else []
    ckpt = os.path.join(a.out_dir, "pretrain.pt")
    if s in ("pretrain", "draft"):
        preset = a.preset if s == "pretrain" else a.draft_preset
        args = ["--data", a.data, "--preset", preset, "--seq_len", str(a.seq_len), "--batch_size",
                str(a.batch_size), "--steps", str(steps), "--out", os.path.join(a.out_dir, f"{s}.pt"),
                "--state_out", os.path.join(a.out_dir, f"{s}_state.pt"),
                "--log_file", os.path.join(a.out_dir, f"{s}_log.jsonl")]
        devs = [d for d in a.devices.split(",") if d]
        if len(devs) > 1:
            cmd = [sys.executable, "-m", "omnicoder.tools.torchrun_ep", "--script", "omnicoder.training.pretrain",
                   "--devices", ",".join(devs), "--"] + args
        else:
            cmd = [sys.executable, "-m", "omnicoder.training.pretrain"] + args
    elif s == "distill":
        cmd = [sys.executable, "-m", "omnicoder.training.distill", "--student_preset", a.draft_preset,
               "--data", a.data, "--steps", str(steps), "--seq_len", str(a.seq_len), "--batch_size",
               str(a.batch_size), "--out", os.path.join(a.out_dir, "student.pt")]
        cmd += (["--teacher_hf", a.teacher_hf] if a.teacher_hf else
                ["--teacher_ckpt", os.path.join(a.out_dir, "pretrain.pt"), "--teacher_preset", a.preset])
    elif s == "draft_kd":
        cmd = [sys.executable, "-m", "omnicoder.training.draft_train", "--student_preset", a.draft_preset,
               "--steps", str(steps), "--seq_len", str(a.seq_len), "--batch_size", str(a.batch_size),
               "--lora", "--out_ckpt", os.path.join(a.out_dir, "draft_kd.pt"),
               "--out_onnx", os.path.join(a.out_dir, "draft_decode_step.onnx"),
               "--bench_out", os.path.join(a.out_dir, "draft_acceptance.json")] + dev
        cmd += (["--teacher_ckpt", ckpt, "--teacher_preset", a.preset] if os.path.exists(ckpt) else
                ["--teacher_preset", a.preset])
    elif s == "code_expert":
        cmd = [sys.executable, "-m", "omnicoder.training.code_expert", "--student_preset", a.preset,
               "--steps", str(steps), "--seq_len", str(a.seq_len), "--batch_size", str(a.batch_size),
               "--data", a.data, "--out", os.path.join(a.out_dir, "code_expert.pt")] + dev
        if os.path.exists(ckpt):
            cmd += ["--teacher_ckpt", ckpt]
    elif s == "verifier":
        cmd = [sys.executable, "-m", "omnicoder.training.verifier_distill", "--student_preset", a.preset,
               "--steps", str(steps), "--seq_len", str(a.seq_len), "--batch_size", str(a.batch_size),
               "--out", os.path.join(a.out_dir, "verifier_kd.pt")] + dev
        if os.path.exists(ckpt):
            cmd += ["--teacher_ckpt", ckpt]
    elif s in ("vl", "vqa"):
        cmd = [sys.executable, "-m", "omnicoder.training.vl_tasks", "--task", "vl_pretrain" if s == "vl" else "vqa",
               "--preset", a.preset, "--steps", str(steps), "--out", os.path.join(a.out_dir, f"{s}.pt")]
        cmd += dev
    elif s == "pre_align":
        cmd = [sys.executable, "-m", "omnicoder.training.pre_align", "--steps", str(steps), "--audio",
               "--out", os.path.join(a.out_dir, "pre_align.pt")] + dev
    elif s == "align":
        pa = os.path.join(a.out_dir, "pre_align.pt")
        cmd = [sys.executable, "-m", "omnicoder.training.concept_align", "--preset", a.preset, "--steps",
               str(steps), "--out", os.path.join(a.out_dir, "concept_head.pt")] + dev
        if os.path.exists(pa):
            cmd += ["--pre_align_ckpt", pa]
    elif s in ("flow_recon", "audio_recon"):
        cmd = [sys.executable, "-m", f"omnicoder.training.{s}", "--preset", a.preset, "--steps",
               str(steps), "--out", os.path.join(a.out_dir, f"{s}_head.pt")] + dev
    elif s == "rl":
        cmd = [sys.executable, "-m", "omnicoder.training.rl", "--preset", a.preset, "--steps", str(steps),
               "--out", os.path.join(a.out_dir, "rl.pt")] + dev
        if os.path.exists(ckpt):
            cmd += ["--ckpt", ckpt]
    elif s == "eval":
        cmd = [sys.executable, "-m", "omnicoder.eval.auto_benchmark", "--preset", a.preset, "--seq_len", "32",
               "--gen_tokens", "8", "--out", os.path.join(a.out_dir, "bench_summary.json")]
        if os.path.exists(ckpt):
            cmd += ["--ckpt", ckpt]
        if a.device:
            cmd += ["--device", a.device]
    elif s == "package":
        cmd = [sys.executable, "-m", "omnicoder.tools.export_to_phone", "--preset", a.preset, "--out",
               os.path.join(a.out_dir, "package")] + (["--ckpt", ckpt] if os.path.exists(ckpt) else [])
    elif s == "export":
        cmd = [sys.executable, "-m", "omnicoder.export.onnx_export", "--ckpt", ckpt,
               "--out", os.path.join(a.out_dir, "decode_step.onnx")]
    else:
        raise SystemExit(f"unknown stage {s}")
    return cmd


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--out_dir", default="weights")
    ap.add_argument("--data", default="synthetic")
    ap.add_argument("--budget_minutes", type=float, default=10.0)
    ap.add_argument("--steps_per_minute", type=float, default=60.0)
    ap.add_argument("--stages", default="pretrain,draft")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--draft_preset", default="draft_2l")
    ap.add_argument("--seq_len", type=int, default=256)
    ap.add_argument("--batch_size", type=int, default=4)
    ap.add_argument("--devices", default="", help="comma list of cuda devices: expert-parallel launch when > 1")
    ap.add_argument("--teacher_hf", default=None, help="distill stage: local Hugging Face causal LM directory")
    ap.add_argument("--smoke_one_step", action="store_true", help="one step per stage (wiring check)")
    ap.add_argument("--device", default="", help="device passed to the stages (default: their own)")
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--dry_run", action="store_true")
    ap.add_argument("--probe", action="store_true",
                    help="measure each stage's steps per minute first and plan with the measured rates")
    ap.add_argument("--probe_only", action="store_true", help="write the probe summary and stop")
    ap.add_argument("--probe_json", default="", help="plan with the rates of an earlier probe summary")
    a = ap.parse_args(argv)
    os.makedirs(a.out_dir, exist_ok=True)
    stages = [s for s in a.stages.split(",") if s]
    rate = a.steps_per_minute
    if a.probe or a.probe_only:
        pr = probe(stages, a)
        with open(os.path.join(a.out_dir, "train_probe_summary.json"), "w") as f:
            json.dump(pr, f, indent=1)
        if a.probe_only:
            print(json.dumps({"probe": pr}, indent=1))
            return 0 if all(v["rc"] == 0 for v in pr.values()) else 1
        rate = {k: v.get("steps_per_minute", 0.0) for k, v in pr.items()}
    elif a.probe_json:
        with open(a.probe_json) as f:
            rate = {k: v.get("steps_per_minute", 0.0) for k, v in json.load(f).items()}
    p = plan(a.budget_minutes, rate, stages)
    if a.smoke_one_step:
        for v in p.values():
            v["steps"] = 1
    results = {}
    for s in stages:
        marker = os.path.join(a.out_dir, f".stage_{s}.done")
        if os.path.exists(marker) and not a.force:
            results[s] = "skipped (done)"
            continue
        cmd = stage_command(s, a, p[s]["steps"])
        if a.dry_run:
            print(" ".join(cmd))
            continue
        t0 = time.time()
        rc = run_with_timeout(cmd, p[s]["minutes"] * 60 * 1.5 + 60)
        results[s] = {"rc": rc, "seconds": round(time.time() - t0, 1)}
        if rc == 0:
            open(marker, "w").close()
        else:
            break
    print(json.dumps({"plan": p, "results": results}, indent=1))
    return 0 if all(not isinstance(v, dict) or v["rc"] == 0 for v in results.values()) else 1


if __name__ == "__main__":
    sys.exit(main())
