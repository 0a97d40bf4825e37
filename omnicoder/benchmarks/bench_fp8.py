"""Block-scaled fp8 GEMMs against the bf16 tcgen05 GEMM and cuBLAS bf16 on the GEMM
shapes of the expert-parallel MoE layer (H 4096, ffn 1408, 8 experts per rank, 8192
tokens x top-6 per rank) and a square 8192^3.

  fp8        block-scaled MMA (kind::mxf8f6f4, power-of-two scales applied by the tensor core)
  fp8_promo  per-K-block partial products promoted by the epilogue (fp32 scales)

    python -m omnicoder.benchmarks.bench_fp8

Times are CUDA-event medians with L2 flushed between calls; the fp8 times are the
GEMM only (operands already quantised); TFLOP/s counts 2 M N K.
"""
from __future__ import annotations

import json

import torch

from omnicoder.benchmarks.timing import time_fn
from omnicoder.ops import _ext, fp8


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--calls", type=int, default=0,
                    help="only run the 8192^3 block-scaled GEMM this many times, untimed (a small case for a profiler)")
    a = ap.parse_args(argv)
    C = _ext.load()
    if a.calls:
        x = torch.randn(8192, 8192, device="cuda").to(torch.bfloat16)
        w = (torch.randn(8192, 8192, device="cuda") * 0.02).to(torch.bfloat16)
        xq, sx = fp8.quantize_act(x)
        wq, sw = fp8.quantize_weight(w)
        out = torch.empty(8192, 8192, device="cuda", dtype=torch.bfloat16)
        for _ in range(a.calls):
            C.fp8_gemm(xq, sx, wq, sw.reshape(-1), out)
        torch.cuda.synchronize()
        _ext.check_status()
        return
    res = []
    for name, M, N, K in [("square_8192", 8192, 8192, 8192), ("expert_gate_up_dense", 6144, 2816, 4096),
                          ("expert_down_dense", 6144, 4096, 1408 // 128 * 128)]:
        x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
        xq, sx = fp8.quantize_act(x)
        wq, sw = fp8.quantize_weight(w)
        pq, ps = fp8.quantize_act(x, pow2=False)
        vq, vs = fp8.quantize_weight(w, pow2=False)
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        t8 = time_fn(lambda: C.fp8_gemm(xq, sx, wq, sw.reshape(-1), out))
        tp = time_fn(lambda: C.fp8_gemm(pq, ps, vq, vs.reshape(-1), out, scaled_mma=False))
        tq = time_fn(lambda: C.fp8_quant_act(x))
        tb = time_fn(lambda: C.gemm(x, w, out, False, False, 0, 1.0, None, None, 256))
        tc = time_fn(lambda: torch.matmul(x, w.t()))
        fl = 2.0 * M * N * K
        res.append({"gemm": name, "M": M, "N": N, "K": K, "fp8_ms": t8, "fp8_tflops": fl / t8 / 1e9,
                    "fp8_promo_ms": tp, "fp8_promo_tflops": fl / tp / 1e9, "act_quant_ms": tq, "bf16_ms": tb, "bf16_tflops": fl / tb / 1e9, "cublas_bf16_ms": tc})
    # grouped: 8 experts x 6144 rows (8192 tokens x top-6 / 8 experts per rank)
    G, rows_per, N, K = 8, 6144, 2816, 4096
    rows = G * rows_per
    off = torch.arange(0, rows + 1, rows_per, dtype=torch.int32, device="cuda")
    x = torch.randn(rows, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(G, N, K, device="cuda") * 0.02).to(torch.bfloat16)
    xq, sx = fp8.quantize_act(x)
    wq, sw = fp8.quantize_weight(w)
    pq, ps = fp8.quantize_act(x, pow2=False)
    vq, vs = fp8.quantize_weight(w, pow2=False)
    out = torch.empty(rows, N, device="cuda", dtype=torch.bfloat16)
    t8 = time_fn(lambda: C.fp8_gemm(xq, sx, wq, sw.reshape(-1), out, off, rows))
    tp = time_fn(lambda: C.fp8_gemm(pq, ps, vq, vs.reshape(-1), out, off, rows, False))
    tb = time_fn(lambda: C.gemm_grouped_m(x, w, off, out, False, 0, 1.0, None, None, 256, rows))
    fl = 2.0 * rows * N * K
    res.append({"gemm": "experts gate|up grouped (8 x 6144 rows)", "M": rows, "N": N, "K": K, "fp8_ms": t8,
                "fp8_tflops": fl / t8 / 1e9, "fp8_promo_ms": tp, "fp8_promo_tflops": fl / tp / 1e9, "bf16_ms": tb, "bf16_tflops": fl / tb / 1e9})
    _ext.check_status()
    for r in res:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
