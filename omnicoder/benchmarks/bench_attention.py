"""Flash-attention forward / backward timing (CUDA events, L2 flushed between runs).

    python -m omnicoder.benchmarks.bench_attention [--batch 2 --seq 4096 --heads 16 --dq 192 --dv 128 --rope]

Default shape: the MLA attention of the moe_mla_24l pretraining model (16 heads,
q/k dim 128 nope + 64 rope, v dim 128, causal, 2 sequences of 4096).  FLOPs
count the causal half: fwd 2 matmuls, bwd 5 (dQ, dK, dV, dP; S recomputed).
"""
from __future__ import annotations

import argparse
import json
import math

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=2)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--kv_heads", type=int, default=0)
    ap.add_argument("--dq", type=int, default=192)
    ap.add_argument("--dv", type=int, default=128)
    ap.add_argument("--rope", type=int, default=64, help="rope part of dq shared by all heads (MLA); 0 = none")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--only", default="", choices=["", "fwd", "bwd"])
    ap.add_argument("--json", default=None)
    a = ap.parse_args(argv)
    from omnicoder.ops import _ext
    C = _ext.load()
    dev = torch.device("cuda")
    T, H = a.batch * a.seq, a.heads
    Hk = a.kv_heads or H
    dk = a.dq - a.rope
    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randn(T, H, a.dq, generator=g).to(dev, torch.bfloat16)
    k = torch.randn(T, Hk, dk, generator=g).to(dev, torch.bfloat16)
    v = torch.randn(T, Hk, a.dv, generator=g).to(dev, torch.bfloat16)
    kr = torch.randn(T, a.rope, generator=g).to(dev, torch.bfloat16) if a.rope else None
    do = torch.randn(T, H, a.dv, generator=g).to(dev, torch.bfloat16)
    scale = 1.0 / math.sqrt(a.dq)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    causal_pairs = a.batch * H * a.seq * (a.seq + 1) / 2
    f_fwd = 2 * causal_pairs * (a.dq + a.dv)
    f_bwd = 2 * causal_pairs * (2 * a.dq + 3 * a.dv)

    def timeit(fn):
        for _ in range(a.warmup):
            fn()
        ts = []
        for _ in range(a.iters):
            flush.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            ts.append(s.elapsed_time(e))
        return sorted(ts)[len(ts) // 2]

    res = {"shape": vars(a)}
    o, lse = C.attn_fwd(q, k, v, kr, a.seq, True, 0, scale)
    if a.only in ("", "fwd"):
        ms = timeit(lambda: C.attn_fwd(q, k, v, kr, a.seq, True, 0, scale))
        res["fwd_ms"], res["fwd_tflops"] = ms, f_fwd / ms / 1e9
    if a.only in ("", "bwd"):
        ms = timeit(lambda: C.attn_bwd(q, k, v, kr, o, lse, do, a.seq, True, 0, scale))
        res["bwd_ms"], res["bwd_tflops"] = ms, f_bwd / ms / 1e9
    _ext.check_status()
    print(json.dumps(res))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
