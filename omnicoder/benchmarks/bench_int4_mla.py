"""Microbenchmarks of the reference's inference bench (src/omnicoder/inference/benchmark.py:
int4-vs-fp32 linear and MLA-vs-SDPA attention), on this package's kernels:

  * weight-only int4 linear (`omnicoder.ops.library.matmul_int4`: the int4 GEMV kernel for
    few rows) against a bf16 linear (this package's GEMM) and an fp32 torch.matmul, on
    decode-shaped projections; GB/s = bytes of the weight format streamed / time;
  * `torch.ops.omnicoder.mla` (the tcgen05 flash-attention kernel over [BH, T, D]) against
    torch's scaled_dot_product_attention on the same bf16 tensors; TFLOP/s counts the
    causal half of 4 * BH * T^2 * D.

    python -m omnicoder.benchmarks.bench_int4_mla [--json out.json]

L2 is flushed before every timed call (CUDA events, median of 10).
"""
from __future__ import annotations

import argparse
import json
import os

import torch
import torch.nn.functional as F

from omnicoder.benchmarks.timing import time_fn


def _peaks():
    p = os.path.join(os.path.dirname(__file__), "..", "..", "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return d["hbm_gbs"], d["bf16_tflops"]
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0


def _t(fn):
    try:
        return time_fn(fn)
    except RuntimeError as e:          # a shape this path rejects: record it, keep measuring
        print(json.dumps({"error": str(e)[:120]}))
        return float("nan")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    a = ap.parse_args(argv)
    from omnicoder.ops import _ext
    from omnicoder.ops.gemm import mm_nt
    from omnicoder.ops.library import matmul_int4, mla
    from omnicoder.quant.int4 import pack_int4
    _ext.load()
    hbm, tflops = _peaks()
    dev = torch.device("cuda")
    rows = []
    for name, M, N, K in [("lm_head", 1, 32000, 2048), ("lm_head", 8, 32000, 2048), ("expert up", 8, 2816, 2048)]:
        w = torch.randn(N, K, device=dev) * 0.02
        packed, scale, _ = pack_int4(w)
        x = torch.randn(M, K, device=dev)
        xb, wb = x.bfloat16(), w.bfloat16()
        t4 = _t(lambda: matmul_int4(xb, packed, scale, None, 7.0))
        tb = _t(lambda: mm_nt(xb, wb))
        tf = _t(lambda: x @ w.t())
        b4, bb, bf = packed.numel() + 4 * N, 2 * N * K, 4 * N * K
        rows.append({"op": f"{name} {M}x{N}x{K}", "int4_ms": t4, "bf16_ms": tb, "fp32_ms": tf,
                     "int4_gbs": b4 / t4 / 1e6, "bf16_gbs": bb / tb / 1e6, "fp32_gbs": bf / tf / 1e6,
                     "int4_frac_of_measured_hbm": b4 / t4 / 1e6 / hbm})
    for BH, T, D in [(64, 1024, 128), (16, 4096, 128), (32, 2048, 64)]:
        q, k, v = (torch.randn(BH, T, D, device=dev, dtype=torch.bfloat16) for _ in range(3))
        tm = _t(lambda: mla(q, k, v, None, True))
        ts = _t(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True))
        fl = 2.0 * BH * T * T * D
        rows.append({"op": f"causal attention BH={BH} T={T} D={D}", "mla_ms": tm, "sdpa_ms": ts,
                     "mla_tflops": fl / tm / 1e9, "sdpa_tflops": fl / ts / 1e9,
                     "mla_frac_of_measured_bf16": fl / tm / 1e9 / tflops})
    for r in rows:
        print(json.dumps(r))
    if a.json:
        with open(a.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
