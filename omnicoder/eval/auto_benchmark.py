"""Evaluation / benchmark sweep: ``python -m omnicoder.eval.auto_benchmark``.

Reference: src/omnicoder/eval/auto_benchmark.py:28-1407 (text tokens/s with KV
quantisation variants and speculative decoding, ONNX provider microbenchmarks,
multiple-choice suites (MMLU, ARC, HellaSwag, TruthfulQA, Winogrande, AGIEval, BBH),
code (HumanEval-style pass@k), VQA / caption / ASR scoring from JSONL, a summary JSON and
CSV).  Each part runs only when its input is given; nothing is downloaded.

  * throughput: greedy decode tokens/s of the model for each requested KV-cache format
    (bf16 / int8 on GPU, the u8 / nf4 grouped formats through the decode-step runner);
    with --speculative a draft preset and its acceptance;
  * multiple choice (any of --mmlu_jsonl, --arc_jsonl, ...): rows {"question", "choices": [...],
    "answer": index or text}; the prediction is the choice with the highest mean token
    log-likelihood given the question;
  * --text: perplexity over windows of a text file;
  * --humaneval_jsonl: rows {"prompt", "tests": [...]} scored with pass@k in the sandbox;
  * --vqa_jsonl / --caption_jsonl / --asr_jsonl: prediction files scored by exact match, BLEU
    and word error rate.
"""
from __future__ import annotations

import argparse
import csv
import json
import math
import os
import time

import torch
import torch.nn.functional as F

MC_SUITES = ("mmlu", "arc", "hellaswag", "truthfulqa", "winogrande", "agieval", "bbh")


def _read_jsonl(path: str, limit: int = 0) -> list[dict]:
    rows = []
    with open(path) as f:
        for line in f:
            if line.strip():
                rows.append(json.loads(line))
                if limit and len(rows) >= limit:
                    break
    return rows


@torch.no_grad()
def choice_loglik(model, tokenizer, context: str, choice: str) -> float:
    """Mean log-probability of the choice's tokens after the context."""
    dev = next(model.parameters()).device
    c_ids = tokenizer.encode(context)
    x_ids = tokenizer.encode(choice) or [0]
    ids = torch.tensor([c_ids + x_ids], device=dev)
    logits = model(ids, all_logits=True)["logits"][0, :-1].float()
    lp = F.log_softmax(logits, -1)
    tgt = ids[0, 1:]
    sel = lp.gather(-1, tgt[:, None]).squeeze(-1)[len(c_ids) - 1:]
    return float(sel.mean())


def evaluate_multiple_choice(model, tokenizer, rows: list[dict]) -> dict:
    correct = 0
    for r in rows:
        choices = r["choices"]
        scores = [choice_loglik(model, tokenizer, r["question"] + " ", c) for c in choices]
        pred = max(range(len(choices)), key=scores.__getitem__)
        ans = r["answer"]
        gold = ans if isinstance(ans, int) else choices.index(ans) if ans in choices else -1
        correct += int(pred == gold)
    return {"accuracy": correct / max(1, len(rows)), "n": len(rows)}


def throughput(model, kv_formats: list[str], seq_len: int, gen: int, batch: int) -> dict:
    from ..inference.benchmark import bench_tokens_per_second
    out = {}
    dev = next(model.parameters()).device
    for kv in kv_formats:
        if kv in ("none", "int8"):
            if kv == "int8" and dev.type != "cuda":
                continue
            out[f"tokens_per_s_kv_{kv}"] = bench_tokens_per_second(model, seq_len=seq_len, gen_tokens=gen,
                                                                   batch=batch, kvq=kv)
        else:                                                   # grouped u8 / nf4 through the step runner
            from ..inference.runtimes import DecodeRunner, TorchStepSession
            import numpy as np
            cpu = model if dev.type == "cpu" else None
            if cpu is None:
                continue
            runner = DecodeRunner(TorchStepSession(cpu, max_len=seq_len + gen + 1, batch=batch), kv_quant=kv)
            prompt = np.random.default_rng(0).integers(0, model.cfg.vocab_size, (batch, seq_len))
            t0 = time.perf_counter()
            runner.generate(prompt, gen)
            out[f"tokens_per_s_kv_{kv}"] = batch * gen / (time.perf_counter() - t0)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description="evaluation and throughput sweep")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--ckpt", default="")
    ap.add_argument("--device", default="auto")
    ap.add_argument("--seq_len", type=int, default=128)
    ap.add_argument("--gen_tokens", type=int, default=64)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--kv", default="none,int8,u8,nf4", help="KV-cache formats to time")
    ap.add_argument("--speculative", action="store_true")
    ap.add_argument("--draft_preset", default="draft_2l")
    ap.add_argument("--mtp", type=int, default=4, help="draft tokens per speculative step")
    ap.add_argument("--text", default="", help="text file for perplexity")
    ap.add_argument("--max_samples", type=int, default=200)
    for s in MC_SUITES:
        ap.add_argument(f"--{s}_jsonl", default="")
    ap.add_argument("--humaneval_jsonl", default="")
    ap.add_argument("--pass_k", type=int, default=1)
    ap.add_argument("--vqa_jsonl", default="", help="rows {prediction, answer}")
    ap.add_argument("--caption_jsonl", default="", help="rows {prediction, references: [...]}")
    ap.add_argument("--asr_jsonl", default="", help="rows {prediction, reference}")
    ap.add_argument("--out", default="weights/bench_summary.json")
    ap.add_argument("--out_csv", default="")
    a = ap.parse_args(argv)
    dev = ("cuda" if torch.cuda.is_available() else "cpu") if a.device == "auto" else a.device
    from ..inference.builders import build_mobile_model_by_name, load_model
    from ..training.tokenizer import get_tokenizer
    if a.ckpt:
        model, _ = load_model(a.ckpt, dev, preset=a.preset)
    else:
        model = build_mobile_model_by_name(a.preset, device=dev)
    model = model.eval()
    tok = get_tokenizer(model.cfg.vocab_size)
    res = {"preset": a.preset, "device": dev, "ckpt": a.ckpt or None}
    res.update(throughput(model, [k for k in a.kv.split(",") if k], a.seq_len, a.gen_tokens, a.batch))
    if a.speculative:
        from ..config import get_preset
        from ..models.lm import build_model
        from ..training.draft_train import acceptance_bench
        dcfg = get_preset(a.draft_preset)
        dcfg.vocab_size = model.cfg.vocab_size
        draft = build_model(dcfg, device=dev, seed=1).eval()
        res["speculative"] = acceptance_bench(model, draft, model.cfg.vocab_size, k=a.mtp, batch=a.batch,
                                              prompt=a.seq_len, gen=a.gen_tokens)
    if a.text:
        from .metrics import perplexity
        ids = torch.tensor(tok.encode(open(a.text).read()))
        S = a.seq_len
        wins = [ids[i:i + S + 1] for i in range(0, max(0, ids.numel() - S - 1), S)][:a.max_samples]
        if wins:
            res["perplexity"] = perplexity(model, wins)
    for s in MC_SUITES:
        p = getattr(a, f"{s}_jsonl")
        if p:
            res[s] = evaluate_multiple_choice(model, tok, _read_jsonl(p, a.max_samples))
    if a.humaneval_jsonl:
        from .metrics import evaluate_code
        res["humaneval"] = evaluate_code(model, tok, _read_jsonl(a.humaneval_jsonl, a.max_samples), k=a.pass_k,
                                         n=max(a.pass_k, 4))
    from .media_metrics import bleu, exact_match_accuracy, word_error_rate
    if a.vqa_jsonl:
        rows = _read_jsonl(a.vqa_jsonl, a.max_samples)
        res["vqa_exact_match"] = exact_match_accuracy([(r["prediction"], r["answer"]) for r in rows])
    if a.caption_jsonl:
        rows = _read_jsonl(a.caption_jsonl, a.max_samples)
        res["caption_bleu"] = bleu([r["prediction"] for r in rows], [r["references"] for r in rows])
    if a.asr_jsonl:
        rows = _read_jsonl(a.asr_jsonl, a.max_samples)
        res["asr_wer"] = sum(word_error_rate(r["reference"], r["prediction"]) for r in rows) / max(1, len(rows))
    os.makedirs(os.path.dirname(os.path.abspath(a.out)) or ".", exist_ok=True)
    with open(a.out, "w") as f:
        json.dump(res, f, indent=1, default=str)
    if a.out_csv:
        flat = {}
        for k, v in res.items():
            if isinstance(v, dict):
                flat.update({f"{k}.{kk}": vv for kk, vv in v.items()})
            else:
                flat[k] = v
        with open(a.out_csv, "w", newline="") as f:
            w = csv.writer(f)
            w.writerow(list(flat))
            w.writerow([flat[k] for k in flat])
    print(json.dumps(res, default=str))
    return 0


if __name__ == "__main__":
    main()
