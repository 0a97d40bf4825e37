"""Memory-bound kernels of the training and decode steps, each timed alone against the
measured HBM copy bandwidth: RMSNorm forward / backward (fused residual add), RoPE,
router top-k, the MoE permutation plan, gather and weighted combine, the int8 KV-cache
append, the int4 weight-only GEMV and the speculative-verification kernel.

    python -m omnicoder.benchmarks.bench_small_kernels [--only rmsnorm,rope,...] [--calls N]

Shapes are those of the moe_mla_24l pretraining step (8192 tokens of d 2048, 16 heads
of q dim 192 with a 64-wide rope part, 32 experts top-4) and of a batch-64 decode step
(MLA latent 512 + 64 int8 KV rows, 4096 x 2048 int4 weights).  Time: CUDA events,
median of `--iters`, L2 flushed before each call; bytes: what the kernel must read and
write once.  `--calls N` instead runs each kernel N times untimed (a small case for a
profiler).
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from omnicoder.benchmarks.timing import time_fn
from omnicoder.ops import _ext


def _peak_gbs() -> float:
    try:
        with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


def cases(dev):
    """name -> (callable, bytes moved once)."""
    C = _ext.load()
    T, D, H, DQ, E, K = 8192, 2048, 16, 192, 32, 4
    bf = torch.bfloat16
    out = {}
    x = torch.randn(T, D, device=dev, dtype=bf)
    r = torch.randn(T, D, device=dev, dtype=bf)
    w = torch.ones(D, device=dev, dtype=bf)
    out["rmsnorm_fwd (residual add)"] = (lambda: C.rmsnorm_fwd(x, r, w, 1e-6), 2 * T * D * 2 + 2 * T * D * 2 + 4 * T)
    y, rstd, h = C.rmsnorm_fwd(x, r, w, 1e-6)
    dy = torch.randn_like(x)
    out["rmsnorm_bwd"] = (lambda: C.rmsnorm_bwd(h, w, rstd, dy, None), 3 * T * D * 2 + 4 * T)
    q = torch.randn(T, H, DQ, device=dev, dtype=bf)
    from omnicoder.ops.layers import RopeTable
    tab = RopeTable(64, 4096, device=dev)
    pos = torch.arange(T, device=dev, dtype=torch.int32) % 4096
    out["rope (q, 16 heads x 64 of 192)"] = (
        lambda: C.rope(q, tab.cs, pos, 0, 4096, T, H, H * DQ, DQ, 128, 64, False, 1.0), 2 * T * H * 64 * 2)
    logits = torch.randn(T, E, device=dev)
    out["router_topk (32 experts, top-4)"] = (lambda: C.router_topk(logits, K, True), T * E * 4 + T * K * 8 + T * E * 4)
    idx = C.router_topk(logits, K, True)[0]
    from omnicoder.ops.moe import cap_rows_for
    rows = cap_rows_for(T, K, E, 0)
    out["moe_plan (count, scan, assign)"] = (lambda: C.moe_plan(idx, E, 0, rows), T * K * 4 * 3 + rows * 4)
    counts, offsets, pos_, src = C.moe_plan(idx, E, 0, rows)
    xp = torch.empty(rows, D, device=dev, dtype=bf)
    out["moe_gather (8192 x top-4 rows)"] = (lambda: C.moe_gather(x, src, xp, K, offsets), 2 * T * K * D * 2)
    wts = torch.rand(T, K, device=dev)
    out["moe_combine (weighted sum + add)"] = (lambda: C.moe_combine(xp, pos_, wts, x), T * K * D * 2 + 2 * T * D * 2)
    # decode: int8 latent KV append for 64 sequences
    Bd, L, G, Dl = 64, 8704, 1, 576
    src_kv = torch.randn(Bd, 1, G, Dl, device=dev, dtype=bf)
    kv = torch.zeros(Bd, L, G, Dl, device=dev, dtype=torch.int8)
    ks = torch.zeros(Bd, L, G, device=dev)
    kpos = torch.full((Bd, 1), 8300, device=dev, dtype=torch.long)
    out["kv_cache_write (int8, 64 x 1 token x 576)"] = (lambda: C.kv_cache_write(src_kv, kpos, kv, ks, 0),
                                                       Bd * Dl * 2 + Bd * Dl + Bd * 4)
    # int4 GEMV: one decode row against a 4096 x 2048 weight (the reference's matmul_int4 shape family)
    from omnicoder.quant.int4 import pack_int4
    N4, K4 = 4096, 2048
    w4 = torch.randn(N4, K4, device=dev) * 0.02
    packed, scale, _ = pack_int4(w4)
    xr = torch.randn(1, K4, device=dev, dtype=bf)
    out["int4_gemv (1 x 2048 @ 4096 x 2048)"] = (lambda: C.int4_gemv(xr, packed, scale, 7.0),
                                                packed.numel() + scale.numel() * 4 + N4 * 2 + K4 * 2)
    # speculative verification: 64 sequences x 4 draft tokens, vocab 32000, sampled (temperature 1)
    Bs, Ks, V = 64, 4, 32000
    lg = torch.randn(Bs, Ks + 1, V, device=dev)
    pd = torch.softmax(torch.randn(Bs, Ks, V, device=dev), -1)
    dr = torch.randint(0, V, (Bs, Ks), device=dev)
    us = torch.rand(Bs, Ks + 1, device=dev)
    bl = torch.full((Bs,), 8192, device=dev, dtype=torch.long)
    out["spec_verify (64 x 4 drafts, vocab 32000)"] = (lambda: C.spec_verify(lg, pd, dr, us, bl, 1.0),
                                                      lg.numel() * 4 + pd.numel() * 4)
    # Gaussian splatting: 4 images of 256 x 256, 65536 Gaussians each, 11 x 11 footprint taps with depth;
    # bytes = the Gaussians' parameters read once and the colour / depth images written once (the
    # 158.6 M accumulator reductions stay in L2)
    Bg, Ng, Hg, Wg, kg = 4, 65536, 256, 256, 11
    gu, gv = torch.rand(Bg, Ng, device=dev) * Wg, torch.rand(Bg, Ng, device=dev) * Hg
    gs = torch.rand(Bg, Ng, device=dev) * 1.5 + 0.5
    go, gz = torch.rand(Bg, Ng, device=dev), torch.rand(Bg, Ng, device=dev) + 1.0
    gc = torch.rand(Bg, Ng, 3, device=dev)
    out["gsplat (4 x 65536 Gaussians, 11 x 11 taps, 256 x 256)"] = (
        lambda: C.gsplat_forward(gu, gv, gs, gs, go, gc, gz, Hg, Wg, kg), Bg * Ng * 9 * 4 + Bg * 4 * Hg * Wg * 4)
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="", help="comma-separated substrings of case names")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--calls", type=int, default=0, help="run each selected kernel N times, untimed, and exit")
    ap.add_argument("--json", default=None)
    a = ap.parse_args(argv)
    dev = torch.device("cuda")
    sel = [s for s in a.only.split(",") if s]
    cs = {k: v for k, v in cases(dev).items() if not sel or any(s in k for s in sel)}
    if a.calls:
        for fn, _ in cs.values():
            for _ in range(a.calls):
                fn()
        torch.cuda.synchronize()
        _ext.check_status()
        return
    peak = _peak_gbs()
    res = []
    for name, (fn, nbytes) in cs.items():
        ms = time_fn(fn, iters=a.iters)
        gbs = nbytes / (ms / 1e3) / 1e9
        res.append({"kernel": name, "us": ms * 1e3, "bytes": nbytes, "gb_s": gbs, "of_measured_hbm": gbs / peak})
    _ext.check_status()
    for r in res:
        print(json.dumps(r))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
