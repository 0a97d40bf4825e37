"""Student-teacher agreement over a prompt set (reference src/omnicoder/eval/teacher_verify.py:1-141:
greedy student outputs compared with each teacher's outputs and with the rows' targets).

Rows are JSONL with `prompt` (or `question`) and optionally `target` (or `answer`).  The student is
this package's model (a checkpoint, or random weights of a preset); a teacher is another checkpoint
of this package (`*.pt`) or a local Hugging Face causal-LM directory (loaded with
local_files_only, so nothing is downloaded).

Agreement of two strings is the partial ratio: the best similarity between the shorter string and
any window of the longer one of the same length, where similarity is difflib's 2 M / T (M matched
characters, T total characters of both); 1.0 when the strings are equal or one contains the other,
otherwise 0.0 when either is empty (two empty outputs count as agreeing, unlike the reference).
The report gives the mean agreement per teacher and the student's mean agreement with the targets.
"""
from __future__ import annotations

import argparse
import difflib
import json
import os

import torch


def partial_ratio(a: str, b: str) -> float:
    a, b = a.strip().lower(), b.strip().lower()
    if a == b:
        return 1.0
    if not a or not b:
        return 0.0
    short, long_ = (a, b) if len(a) <= len(b) else (b, a)
    if short in long_:
        return 1.0
    n = len(short)
    m = difflib.SequenceMatcher(None, short, long_, autojunk=False)
    best = 0.0
    # windows aligned with each matching block are the only ones that can score best
    for blk in m.get_matching_blocks():
        start = max(0, min(blk.b - blk.a, len(long_) - n))
        r = difflib.SequenceMatcher(None, short, long_[start:start + n], autojunk=False).ratio()
        best = max(best, r)
    return best


def read_rows(path: str, limit: int = 0) -> list[dict]:
    rows = []
    with open(path, encoding="utf-8", errors="replace") as f:
        for line in f:
            if line.strip():
                rows.append(json.loads(line))
                if limit and len(rows) >= limit:
                    break
    return rows


@torch.no_grad()
def omni_generate(model, tok, prompts: list[str], max_new_tokens: int) -> list[str]:
    from ..inference.generate import generate
    dev = next(model.parameters()).device
    outs = []
    for p in prompts:
        ids = torch.tensor([tok.encode(p) or [1]], dtype=torch.long, device=dev)
        y = generate(model, ids, max_new_tokens, temperature=0.0, cuda_graph=False)
        outs.append(tok.decode(y[0, ids.shape[1]:].tolist()))
    return outs


@torch.no_grad()
def hf_generate(path: str, prompts: list[str], max_new_tokens: int, device: str = "cpu") -> list[str]:
    from transformers import AutoModelForCausalLM, AutoTokenizer
    tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
    model = AutoModelForCausalLM.from_pretrained(path, local_files_only=True).to(device).eval()
    outs = []
    for p in prompts:
        enc = tok(p, return_tensors="pt").to(device)
        y = model.generate(**enc, max_new_tokens=max_new_tokens, do_sample=False)
        outs.append(tok.decode(y[0, enc["input_ids"].shape[1]:], skip_special_tokens=True))
    return outs


def agreement_report(rows: list[dict], student_out: list[str], teacher_outs: dict[str, list[str]]) -> dict:
    res = {"samples": len(rows), "teachers": {}, "overall": {}}
    for name, outs in teacher_outs.items():
        sc = [partial_ratio(s, o) for s, o in zip(student_out, outs)]
        res["teachers"][name] = {"agreement": sum(sc) / max(1, len(sc))}
    targets = [str(r.get("target") or r.get("answer") or "") for r in rows]
    sc = [partial_ratio(s, t) for s, t in zip(student_out, targets) if t]
    if sc:
        res["overall"]["student_vs_target"] = sum(sc) / len(sc)
    if res["teachers"]:
        res["overall"]["mean_teacher_agreement"] = (sum(v["agreement"] for v in res["teachers"].values())
                                                    / len(res["teachers"]))
    return res


def main(argv=None):
    from ..config import get_preset
    from ..inference.builders import load_model
    from ..models.lm import build_model
    from ..training.tokenizer import get_tokenizer
    ap = argparse.ArgumentParser(description="student-teacher agreement over a JSONL prompt set")
    ap.add_argument("--data", required=True)
    ap.add_argument("--domain", default="text", choices=["text", "code"])
    ap.add_argument("--teachers", default="", help="space-separated checkpoints (.pt) or local HF model dirs")
    ap.add_argument("--student_ckpt", default="")
    ap.add_argument("--student_preset", default="tiny_moe")
    ap.add_argument("--max_new_tokens", type=int, default=32)
    ap.add_argument("--limit", type=int, default=64)
    ap.add_argument("--out", default="weights/teacher_verify.json")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dev = torch.device(a.device)
    rows = read_rows(a.data, a.limit)
    prompts = [str(r.get("prompt") or r.get("question") or "") for r in rows]
    student = (load_model(a.student_ckpt, dev)[0] if a.student_ckpt else
               build_model(get_preset(a.student_preset), device=dev, seed=0)).eval()
    tok = get_tokenizer(student.cfg.vocab_size)
    s_out = omni_generate(student, tok, prompts, a.max_new_tokens)
    t_outs = {}
    for t in a.teachers.split():
        if t.endswith(".pt"):
            tm = load_model(t, dev)[0].eval()
            t_outs[t] = omni_generate(tm, get_tokenizer(tm.cfg.vocab_size), prompts, a.max_new_tokens)
        else:
            t_outs[t] = hf_generate(t, prompts, a.max_new_tokens, str(dev))
    res = agreement_report(rows, s_out, t_outs)
    res["domain"] = a.domain
    os.makedirs(os.path.dirname(a.out) or ".", exist_ok=True)
    with open(a.out, "w", encoding="utf-8") as f:
        json.dump(res, f, indent=1)
    print(json.dumps(res))
    return 0


if __name__ == "__main__":
    main()
