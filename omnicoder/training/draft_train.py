"""Draft-model pipeline for speculative decoding: distil, export, measure acceptance.

    python -m omnicoder.training.draft_train [--teacher_ckpt T.pt | --teacher_preset P | --teacher_hf DIR]
        [--student_preset draft_2l] [--steps N] [--lora] [--out_ckpt ...] [--out_onnx ...]

Reference: src/omnicoder/training/draft_train.py:1-130 (KD of a compact student from a
teacher, optional LoRA, one-step ONNX export of the draft, acceptance benchmark).
Stages, all in one process:
  1. knowledge distillation of the student (omnicoder.training.distill.kd_loss; LoRA
     adapters on the student's linear layers with --lora);
  2. checkpoint of the draft (config embedded) and, when `onnx` is installed, its
     decode-step graph (omnicoder.export.onnx_export);
  3. acceptance: speculative decoding of random prompts with the draft against the teacher
     (when the teacher is an omnicoder model): draft acceptance rate, target-only and
     speculative tokens/s, written to --bench_out.
"""
from __future__ import annotations

import argparse
import json
import os
import time

import torch


def acceptance_bench(target, draft, vocab: int, k: int = 4, batch: int = 4, prompt: int = 32, gen: int = 32,
                     seed: int = 0) -> dict:
    """Greedy speculative decoding of random prompts: acceptance rate and tokens/s against plain decoding."""
    from ..inference.generate import generate
    dev = next(target.parameters()).device
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, vocab, (batch, prompt), generator=g).to(dev)
    t0 = time.perf_counter()
    plain = generate(target, ids, gen, temperature=0.0)
    t_plain = time.perf_counter() - t0
    t0 = time.perf_counter()
    spec, st = generate(target, ids, gen, temperature=0.0, draft_model=draft, speculative_draft_len=k,
                        return_stats=True)
    t_spec = time.perf_counter() - t0
    return {"acceptance": st.accepted_draft_tokens / max(1, st.proposed_draft_tokens), "draft_len": k,
            "plain_tokens_per_s": batch * gen / t_plain, "speculative_tokens_per_s": batch * gen / t_spec,
            "same_output": bool(torch.equal(plain, spec))}


def main(argv=None):
    from ..config import TrainConfig, get_preset
    from ..models.lm import build_model
    from .data import SyntheticTokens, batches
    from .distill import kd_loss

    ap = argparse.ArgumentParser(description="distil a draft model, export it, measure its acceptance")
    ap.add_argument("--teacher_ckpt", default=None)
    ap.add_argument("--teacher_preset", default="tiny_moe")
    ap.add_argument("--teacher_hf", default=None, help="local Hugging Face causal LM directory")
    ap.add_argument("--student_preset", default="draft_2l")
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--seq_len", type=int, default=128)
    ap.add_argument("--batch_size", type=int, default=4)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--temperature", type=float, default=2.0)
    ap.add_argument("--alpha", type=float, default=0.9)
    ap.add_argument("--lora", action="store_true", help="train LoRA adapters instead of all student weights")
    ap.add_argument("--lora_r", type=int, default=16)
    ap.add_argument("--lora_alpha", type=int, default=32)
    ap.add_argument("--out_ckpt", default="weights/draft_kd.pt")
    ap.add_argument("--out_onnx", default="weights/draft_decode_step.onnx")
    ap.add_argument("--bench_out", default="weights/draft_acceptance.json")
    ap.add_argument("--draft_len", type=int, default=4)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dev = torch.device(a.device)
    # ---- teacher -------------------------------------------------------------------------------
    if a.teacher_hf:
        from transformers import AutoModelForCausalLM
        teacher = AutoModelForCausalLM.from_pretrained(a.teacher_hf, local_files_only=True).to(dev).eval()
        vocab = teacher.config.vocab_size
    else:
        if a.teacher_ckpt:
            from ..inference.builders import load_model
            teacher, _ = load_model(a.teacher_ckpt, dev, preset=a.teacher_preset)
        else:
            teacher = build_model(get_preset(a.teacher_preset), device=dev, seed=0)
        teacher = teacher.eval()
        vocab = teacher.cfg.vocab_size
    # ---- student ---------------------------------------------------------------------------------
    scfg = get_preset(a.student_preset)
    scfg.vocab_size = vocab
    student = build_model(scfg, device=dev, seed=1)
    if a.lora:
        from .lora import inject_lora
        inject_lora(student, r=a.lora_r, alpha=a.lora_alpha)
    params = [p for p in student.parameters() if p.requires_grad]
    opt = torch.optim.AdamW(params, lr=a.lr)
    it = batches(SyntheticTokens(vocab, a.seq_len, seed=0), a.batch_size)
    from .distill import _logits
    losses = []
    for _ in range(a.steps):
        ids, lab = next(it)
        ids, lab = ids.to(dev), lab.to(dev)
        with torch.no_grad():
            t = _logits(teacher, ids)
        loss = kd_loss(_logits(student, ids), t, lab, a.temperature, a.alpha)
        loss.backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        losses.append(float(loss))
    if a.lora:
        from .lora import merge_lora
        merge_lora(student)
    os.makedirs(os.path.dirname(os.path.abspath(a.out_ckpt)) or ".", exist_ok=True)
    torch.save({"model": student.export_state_dict(), "config": student.cfg.to_dict(), "step": a.steps},
               a.out_ckpt)
    report = {"kd_first_loss": losses[0] if losses else None, "kd_last_loss": losses[-1] if losses else None,
              "ckpt": a.out_ckpt}
    try:
        from ..export.onnx_export import export_decode_step
        cpu_student = build_model(student.cfg, device="cpu", dtype=torch.float32, seed=None)
        cpu_student.load_state_dict({k: v.float().cpu() for k, v in student.state_dict().items()})
        export_decode_step(cpu_student.eval(), a.out_onnx)
        report["onnx"] = a.out_onnx
    except RuntimeError as e:
        report["onnx"] = f"skipped: {e}"
    if not a.teacher_hf:
        report["acceptance"] = acceptance_bench(teacher, student.eval(), vocab, k=a.draft_len)
    os.makedirs(os.path.dirname(os.path.abspath(a.bench_out)) or ".", exist_ok=True)
    with open(a.bench_out, "w") as f:
        json.dump(report, f, indent=1)
    print(json.dumps(report))
    return 0


if __name__ == "__main__":
    main()
