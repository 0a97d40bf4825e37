"""Long-context batched inference benchmark: prefill tokens/s, decode tokens/s and
time per output token, optionally with speculative decoding.

    python -m omnicoder.benchmarks.bench_inference [--batch 64 --prompt 8192 --gen 512 --kv int8 --spec 4]

Default workload: the longctx_moe model (the 24-layer MLA MoE architecture of
the pretraining benchmark, sliding window 4096 + 64 compressed memory rows),
int8 latent KV cache (one scale per token), 64 random prompts of 8192 tokens,
512 generated tokens; speculative decoding with the 2-layer d1024 draft model
proposing 4 tokens per step, verified by the target in one forward.  Weights are
random (N(0, 0.02)), so draft acceptance is what random weights give.
Timing: CUDA events around prefill and around every decode step (the device
time of the step; the host reads the sampled ids each step, as a server would).
"""
from __future__ import annotations

import argparse
import json
import statistics

import torch

from omnicoder.config import get_preset
from omnicoder.inference.kv_cache import KVCache
from omnicoder.models.lm import build_model
from omnicoder.ops import _ext
from omnicoder.ops.spec import spec_verify


def run(preset="longctx_moe", draft_preset="draft_2l", batch=64, prompt=8192, gen=512, kv="int8", spec=0,
        prefill_chunk=4, layers=0, graphs=True, seed=0, device=None, profile_steps=0, parallel=None):
    """One long-context batched generation; returns the result dict (device-timed with CUDA events).
    `parallel` (omnicoder.parallel.expert_data.ExpertDataParallel): the routed experts are sharded
    over its ranks (expert parallel); every rank serves its own `batch` sequences with its own KV
    cache and all ranks run this function together."""
    dev = device or torch.device("cuda")
    _ext.load()
    cfg = get_preset(preset)
    if layers:
        cfg.n_layers = layers
    cfg.max_seq_len = max(cfg.max_seq_len, prompt + gen + spec + 1)
    # expert parallel: every rank builds the same model (its slice of the experts); prompts differ
    model = build_model(cfg, device=dev, seed=0 if parallel is not None else seed,
                        ep=parallel).eval().prepare_inference()
    draft = None
    if spec > 0:
        dcfg = get_preset(draft_preset)
        dcfg.vocab_size = cfg.vocab_size
        dcfg.max_seq_len = cfg.max_seq_len
        draft = build_model(dcfg, device=dev, seed=seed + 1).eval()
    g = torch.Generator().manual_seed(seed)
    prompts = torch.randint(0, cfg.vocab_size, (batch, prompt), generator=g).to(dev)
    L = prompt + gen + spec + 1
    cache = KVCache(cfg, batch, L, dev, kv_dtype=kv)
    dcache = KVCache(draft.cfg, batch, L, dev) if draft is not None else None
    ev = lambda: torch.cuda.Event(enable_timing=True)
    # the few-row projections may run on the library GEMM: create its handle and workspace before
    # the timed region (a one-time process cost, not part of a prefill)
    with torch.no_grad():
        torch.mm(torch.zeros(8, 64, device=dev, dtype=torch.bfloat16), torch.zeros(64, 8, device=dev,
                                                                                   dtype=torch.bfloat16))
    # ---- prefill: the whole prompt, in chunks of sequences; its last logits give token 1
    torch.cuda.synchronize()
    e0, e1 = ev(), ev()
    e0.record()
    first = []
    with torch.no_grad():
        for b0 in range(0, batch, prefill_chunk):
            b1 = min(batch, b0 + prefill_chunk)
            lg = model.forward_cached(prompts[b0:b1], cache.view(b0, b1), prefill=True, last_only=True)
            first.append(lg[:, -1].argmax(-1))
            if draft is not None:
                draft.forward_cached(prompts[b0:b1], dcache.view(b0, b1), prefill=True, last_only=True)
        n_mem = cache.compress_memory(cfg.attn.window) if cfg.attn.window else 0
        last = torch.cat(first)
    e1.record()
    torch.cuda.synchronize()
    prefill_s = e0.elapsed_time(e1) / 1000.0
    # ---- decode: the remaining gen - 1 tokens ---------------------------------------
    step_ms, produced, accepted, proposed = [], 1, 0, 0
    per_seq = torch.ones(batch, dtype=torch.long, device=dev)       # tokens produced per sequence
    total_new = 0
    fwd_t = lambda ids: model.forward_cached(ids, cache)
    fwd_d = (lambda ids: draft.forward_cached(ids, dcache)) if draft is not None else None
    if graphs:
        from omnicoder.inference.graphs import GraphedStep
        fwd_t = GraphedStep(model, cache, 1 if draft is None else spec + 1)
        if draft is not None:
            fwd_d = GraphedStep(draft, dcache, 1)
    with torch.no_grad():
        ar = torch.arange(batch, device=dev)
        while produced < gen:
            s0, s1 = ev(), ev()
            s0.record()
            if draft is None:
                last = fwd_t(last[:, None])[:, -1].argmax(-1)
                n_new = 1
                total_new += batch
            else:
                base_t, base_d = cache.lengths.clone(), dcache.lengths.clone()
                cur, props = last, []
                for _ in range(spec):
                    cur = fwd_d(cur[:, None])[:, -1].argmax(-1)
                    props.append(cur)
                props = torch.stack(props, 1)                                    # [B, k] proposals
                tl = fwd_t(torch.cat([last[:, None], props], 1))                 # [B, k+1, V]
                # verify kernel: every sequence keeps its own accepted prefix and the target's
                # next token; both caches roll back per sequence (the draft first appends its last
                # proposal, which only fully accepted sequences keep)
                n_acc, last, new_len = spec_verify(tl, None, props, None, base_t, 0.0)
                n_acc = n_acc.long()
                fwd_d(props[:, -1:])
                cache.rollback(new_len)
                dcache.rollback(base_d + n_acc + 1)
                gained = torch.minimum(n_acc + 1, (gen - per_seq).clamp_min(0))
                per_seq += n_acc + 1
                accepted += int(n_acc.sum())
                proposed += batch * spec
                total_new += int(gained.sum())
                n_new = int(per_seq.min()) - produced
            s1.record()
            s1.synchronize()
            step_ms.append(s0.elapsed_time(s1))
            produced += n_new
    _ext.check_status()
    breakdown = _profile_decode(fwd_t, last, profile_steps) if profile_steps and draft is None else None
    decode_s = sum(step_ms) / 1000.0
    res = {
        "metric": "long-context MoE inference (prefill tokens/s, decode tokens/s, p50 TPOT)",
        "model": f"{cfg.name}: {cfg.n_layers}L d{cfg.d_model} MLA kv{cfg.attn.kv_lora_rank} {cfg.moe.n_experts} experts "
                 f"top-{cfg.moe.top_k}, window {cfg.attn.window} + {cfg.attn.mem_slots} memory rows",
        "batch": batch, "prompt": prompt, "gen": gen, "kv": kv, "spec_tokens": spec,
        "prefill_tokens_per_s": batch * prompt / prefill_s, "prefill_s": prefill_s,
        "decode_tokens_per_s": total_new / decode_s, "decode_steps": len(step_ms),
        "p50_step_ms": statistics.median(step_ms),
        "p50_tpot_ms": statistics.median(step_ms) * len(step_ms) * batch / max(1, total_new),
        "expert_parallel": parallel.world if parallel is not None else 1,
        "memory_rows": n_mem, "kv_cache_gb": cache.nbytes() / 1e9,
        "draft_acceptance": (accepted / proposed) if proposed else None, "cuda_graphs": graphs,
        "speculative_acceptance": "per sequence (own accepted prefix and cache rollback)" if spec else None,
        "decode_kernel_breakdown_ms_per_step": breakdown,
        "data": "synthetic (uniform random prompts, random-init N(0,0.02) weights)", "dtype": "bf16 weights",
    }
    return res


def _profile_decode(step, last, n):
    """Kernel time per family over n more decode steps (PyTorch profiler; shares, not a bench number)."""
    import collections

    from torch.profiler import ProfilerActivity, profile

    from omnicoder.benchmarks.profile_step import family
    with torch.no_grad(), profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(n):
            last = step(last[:, None])[:, -1].argmax(-1)
        torch.cuda.synchronize()
    agg = collections.defaultdict(float)
    for e in prof.events():
        if e.device_type is not None and str(e.device_type).endswith("CUDA"):
            agg[family(e.name)] += (e.device_time_total if hasattr(e, "device_time_total") else e.cuda_time_total) / 1e3
    return {k: round(v / n, 4) for k, v in sorted(agg.items(), key=lambda kv: -kv[1])}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="longctx_moe")
    ap.add_argument("--draft", default="draft_2l")
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=8192)
    ap.add_argument("--gen", type=int, default=512)
    ap.add_argument("--kv", default="int8", choices=["int8", "bf16"])
    ap.add_argument("--spec", type=int, default=0, help="draft tokens per step (0: plain decode)")
    ap.add_argument("--prefill_chunk", type=int, default=4, help="sequences per prefill call")
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (quick runs only)")
    ap.add_argument("--no-graphs", dest="graphs", action="store_false", help="run decode steps eagerly")
    ap.add_argument("--json", default=None)
    ap.add_argument("--profile", type=int, default=0, help="profile this many extra decode steps (kernel shares)")
    a = ap.parse_args(argv)
    res = run(a.preset, a.draft, a.batch, a.prompt, a.gen, a.kv, a.spec, a.prefill_chunk, a.layers, a.graphs,
              profile_steps=a.profile)
    print(json.dumps(res))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
