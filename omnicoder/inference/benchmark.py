"""Generation throughput measurement (reference src/omnicoder/inference/benchmark.py:42:
`bench_tokens_per_second`) and a batched decode benchmark.

`bench_tokens_per_second(model, seq_len, gen_tokens, ...)` -> tokens per second of
`generate()` (warm-up first, device-synchronised timing).  `decode_benchmark`
measures prefill and decode separately for a batch of random prompts and
reports tokens/s and the p50 / p90 time per output token.
"""
from __future__ import annotations

import statistics
import time

import torch

from .generate import generate


def _sync(dev):
    if torch.device(dev).type == "cuda":
        torch.cuda.synchronize(dev)


@torch.no_grad()
def bench_tokens_per_second(model, seq_len: int = 128, gen_tokens: int = 128, device=None, batch: int = 1,
                            warmup: int = 1, kvq: str = "none", seed: int = 0, **gen_kw) -> float:
    dev = device or next(model.parameters()).device
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, model.cfg.vocab_size, (batch, seq_len), generator=g).to(dev)
    for _ in range(warmup):
        generate(model, ids, min(gen_tokens, 8), temperature=0.0, kvq=kvq, **gen_kw)
    _sync(dev)
    t0 = time.perf_counter()
    generate(model, ids, gen_tokens, temperature=0.0, kvq=kvq, **gen_kw)
    _sync(dev)
    return batch * gen_tokens / (time.perf_counter() - t0)


@torch.no_grad()
def decode_benchmark(model, batch: int, prompt_len: int, gen_tokens: int, kvq: str = "none", draft=None,
                     spec_tokens: int = 0, seed: int = 0, warmup_tokens: int = 4) -> dict:
    dev = next(model.parameters()).device
    g = torch.Generator().manual_seed(seed)
    ids = torch.randint(0, model.cfg.vocab_size, (batch, prompt_len), generator=g).to(dev)
    generate(model, ids[:, :min(prompt_len, 128)], warmup_tokens, temperature=0.0, kvq=kvq, draft_model=draft,
             speculative_draft_len=spec_tokens)
    _sync(dev)
    out, st = generate(model, ids, gen_tokens, temperature=0.0, kvq=kvq, draft_model=draft,
                       speculative_draft_len=spec_tokens, return_stats=True)
    tpot = sorted(st.step_times_s) or [st.decode_s / max(1, st.steps)]
    per_tok = [t / (1 + (spec_tokens if draft is not None else 0)) for t in tpot]
    return {"batch": batch, "prompt_len": prompt_len, "gen_tokens": gen_tokens,
            "prefill_tokens_per_s": batch * prompt_len / max(st.prefill_s, 1e-9),
            "decode_tokens_per_s": st.new_tokens / max(st.decode_s, 1e-9),
            "p50_tpot_ms": 1000 * statistics.median(tpot), "p90_tpot_ms": 1000 * tpot[int(0.9 * (len(tpot) - 1))],
            "accepted_draft_tokens": st.accepted_draft_tokens, "proposed_draft_tokens": st.proposed_draft_tokens,
            "per_token_ms_est": 1000 * statistics.median(per_tok)}
