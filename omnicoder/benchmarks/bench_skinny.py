"""Few-row (decode-shaped) GEMMs: the swap-AB tcgen05 kernel against the tile
GEMM of this package and against cuBLAS (torch.matmul), on the projections of
one batch-64 decode step of the long-context MoE model (24L d2048, MLA latent
512 + rope 64, 16 heads, 32 experts of ffn 1408, top-4, vocab 32000).

    python -m omnicoder.benchmarks.bench_skinny [--json out.json]
    python -m omnicoder.benchmarks.bench_skinny --grouped-calls 3   # only 3 grouped gate|up calls (for ncu)

L2 is flushed before every timed call, so each call streams its weight matrix
from HBM; reported GB/s = weight bytes / time.
"""
from __future__ import annotations

import argparse
import json

import torch

from omnicoder.benchmarks.timing import time_fn
from omnicoder.ops import _ext

EPI_BF16, EPI_F32, EPI_ACC, EPI_ADD, EPI_SWIGLU = range(5)

DENSE = [
    # name, rows, N, K
    ("q_absorbed (wq_abs)", 64, 16 * 576, 2048),
    ("out_absorbed (wo_abs)", 64, 2048, 16 * 512),
    ("kv_a (wkv_a)", 64, 576, 2048),
    ("lm_head", 64, 32000, 2048),
    ("shared expert gate|up", 64, 2816, 2048),
]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    ap.add_argument("--grouped-calls", type=int, default=0,
                    help="run only this many untimed grouped gate|up calls (a small case for a profiler)")
    a = ap.parse_args(argv)
    C = _ext.load()
    dev = torch.device("cuda")
    res = []
    for name, M, N, K in ([] if a.grouped_calls else DENSE):
        x = torch.randn(M, K, device=dev).to(torch.bfloat16)
        w = (torch.randn(N, K, device=dev) * 0.02).to(torch.bfloat16)
        out = torch.empty(M, N, device=dev, dtype=torch.bfloat16)
        ours = lambda: C.gemm(x, w, out, False, False, EPI_BF16, 1.0, None, None, 256)
        t_sk = time_fn(ours)
        C.set_skinny_rows(0)
        t_tile = time_fn(ours)
        C.set_skinny_rows(128)
        t_cublas = time_fn(lambda: torch.matmul(x, w.t()))
        gb = N * K * 2 / 1e9
        res.append({"gemm": name, "rows": M, "N": N, "K": K, "skinny_us": t_sk * 1e3, "tile_us": t_tile * 1e3,
                    "cublas_us": t_cublas * 1e3, "skinny_gbs": gb / (t_sk / 1e3)})
    # grouped experts of one decode step: 64 tokens x top-4 = 256 rows over 32 experts
    E, D, F, rows = 32, 2048, 1408, 256
    g = torch.Generator(device="cpu").manual_seed(0)
    counts = torch.multinomial(torch.ones(E), rows, replacement=True, generator=g).bincount(minlength=E)
    off = torch.cat([torch.zeros(1, dtype=torch.long), counts.cumsum(0)]).to(torch.int32).to(dev)
    x = torch.randn(rows, D, device=dev).to(torch.bfloat16)
    w13 = (torch.randn(E, 2 * F, D, device=dev) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(E, D, F, device=dev) * 0.02).to(torch.bfloat16)
    act = torch.empty(rows, F, device=dev, dtype=torch.bfloat16)
    y = torch.empty(rows, D, device=dev, dtype=torch.bfloat16)
    if a.grouped_calls:
        for _ in range(a.grouped_calls):
            C.gemm_skinny_grouped(x, w13, off, act, EPI_SWIGLU, 1.0, rows)
        torch.cuda.synchronize()
        _ext.check_status()
        return
    t13 = time_fn(lambda: C.gemm_skinny_grouped(x, w13, off, act, EPI_SWIGLU, 1.0, rows))
    t2 = time_fn(lambda: C.gemm_skinny_grouped(act, w2, off, y, EPI_BF16, 1.0, rows))
    # cuBLAS reference of the same work: one matmul per expert
    segs = [(int(off[e]), int(off[e + 1])) for e in range(E)]
    t_cub = time_fn(lambda: [torch.matmul(x[s:t], w13[e].t()) for e, (s, t) in enumerate(segs)])
    res.append({"gemm": "experts gate|up + SwiGLU (grouped, 256 rows / 32 experts)", "rows": rows, "N": 2 * F, "K": D,
                "skinny_us": t13 * 1e3, "cublas_per_expert_loop_us": t_cub * 1e3,
                "skinny_gbs": E * 2 * F * D * 2 / 1e9 / (t13 / 1e3)})
    res.append({"gemm": "experts down (grouped)", "rows": rows, "N": D, "K": F, "skinny_us": t2 * 1e3,
                "skinny_gbs": E * F * D * 2 / 1e9 / (t2 / 1e3)})
    _ext.check_status()
    for r in res:
        print(json.dumps(r))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    main()
