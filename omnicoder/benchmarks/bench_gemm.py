"""tcgen05 GEMM vs cuBLAS (torch.matmul) on the linear-layer shapes of the
MoE pretraining config (8192 tokens per GPU, d_model 2048, MLA, ffn 1408).

Usage: python -m omnicoder.benchmarks.bench_gemm [--json out.json]
"""
from __future__ import annotations

import argparse
import json

import torch

from omnicoder.benchmarks.timing import time_fn
from omnicoder.ops import _ext

EPI_BF16, EPI_F32, EPI_ACC, EPI_ADD, EPI_SWIGLU, EPI_SWIGLU_BWD = range(6)

SHAPES = [
    # name, M, N, K, kind
    ("square_8192", 8192, 8192, 8192, "fwd"),
    ("q_proj_fwd", 8192, 3072, 2048, "fwd"),
    ("o_proj_fwd", 8192, 2048, 2048, "fwd"),
    ("kv_b_fwd", 8192, 4096, 512, "fwd"),
    ("lm_head_fwd", 8192, 32000, 2048, "fwd"),
    ("shared_gate_up_swiglu", 8192, 2816, 2048, "swiglu"),
    ("o_proj_dx", 8192, 2048, 2048, "dx"),
    ("o_proj_dw", 8192, 2048, 2048, "dw"),
    ("lm_head_dx", 8192, 2048, 32000, "dx"),
    ("expert_w13_dw_grouped", 2816, 2048, 32768, "dw_grouped"),   # 32 experts x 1024 rows
]


def run(shape):
    name, M, N, K, kind = shape
    C = _ext.load()
    a = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    if kind in ("fwd", "swiglu"):
        b = torch.randn(N, K, device="cuda").to(torch.bfloat16) * 0.02
        out = torch.empty(M, N // 2 if kind == "swiglu" else N, device="cuda", dtype=torch.bfloat16)
        H = torch.empty(M, N, device="cuda", dtype=torch.bfloat16) if kind == "swiglu" else None
        epi = EPI_SWIGLU if kind == "swiglu" else EPI_BF16
        ours = lambda: C.gemm(a, b, out, False, False, epi, 1.0, None, H, 256)
        ref = lambda: torch.matmul(a, b.t())
        flops = 2 * M * N * K
    elif kind == "dx":
        # dX[M,N] = dY[M,K] @ W[K,N]
        b = torch.randn(K, N, device="cuda").to(torch.bfloat16) * 0.02
        out = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ours = lambda: C.gemm(a, b, out, False, True, EPI_BF16, 1.0, None, None, 256)
        ref = lambda: torch.matmul(a, b)
        flops = 2 * M * N * K
    elif kind == "dw_grouped":
        # per expert g: dW[g] [M, N] = A_g^T B_g over the expert's rows (K = all rows of 32 experts)
        G = 32
        a = torch.randn(K, M, device="cuda").to(torch.bfloat16)
        b = torch.randn(K, N, device="cuda").to(torch.bfloat16)
        offs = torch.arange(0, K + 1, K // G, device="cuda", dtype=torch.int32)
        out = torch.empty(G, M, N, device="cuda", dtype=torch.bfloat16)
        ours = lambda: C.gemm_grouped_k(a, b, offs, out, EPI_BF16, 1.0, 256)
        ref = lambda: torch.bmm(a.view(G, K // G, M).transpose(1, 2), b.view(G, K // G, N))
        flops = 2 * M * N * K
    else:  # dw: dW[N,K] = dY[M,N]^T X[M,K]
        dy = torch.randn(M, N, device="cuda").to(torch.bfloat16)
        out = torch.empty(N, K, device="cuda", dtype=torch.bfloat16)
        ours = lambda: C.gemm(dy, a, out, True, True, EPI_BF16, 1.0, None, None, 256)
        ref = lambda: torch.matmul(dy.t(), a)
        flops = 2 * M * N * K
    t_ours = time_fn(ours)
    C.set_gemm_pair(False)           # the one-CTA 128-row tile kernel, for comparison
    try:
        t_single = time_fn(ours)
    finally:
        C.set_gemm_pair(True)
    t_ref = time_fn(ref)
    _ext.check_status()
    return {"name": name, "M": M, "N": N, "K": K, "kind": kind, "ms": t_ours, "single_cta_ms": t_single,
            "cublas_ms": t_ref, "tflops": flops / t_ours / 1e9, "single_cta_tflops": flops / t_single / 1e9,
            "cublas_tflops": flops / t_ref / 1e9, "speedup": t_ref / t_ours}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", default=None)
    ap.add_argument("--only", default=None)
    args = ap.parse_args()
    rows = []
    for s in SHAPES:
        if args.only and args.only not in s[0]:
            continue
        r = run(s)
        rows.append(r)
        print(f"{r['name']:24s} M={r['M']:6d} N={r['N']:6d} K={r['K']:6d}  ours {r['ms']:8.3f} ms "
              f"{r['tflops']:7.1f} TF/s (one-CTA tiles {r['single_cta_tflops']:7.1f}) | cuBLAS {r['cublas_ms']:8.3f} ms {r['cublas_tflops']:7.1f} TF/s | x{r['speedup']:.2f}",
              flush=True)
    if args.json:
        with open(args.json, "w") as f:
            json.dump(rows, f, indent=1)


if __name__ == "__main__":
    main()
