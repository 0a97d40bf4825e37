"""One routed MoE FFN layer on one GPU, forward + backward, at the pretraining
shape (8192 tokens, d_model 2048, 32 SwiGLU experts of ffn 1408, top-4,
capacity factor 1.25): router, permutation plan, gather, grouped expert GEMMs
with fused SwiGLU epilogues, combine, and their backward.

    python -m omnicoder.benchmarks.bench_moe_ffn [--tokens 8192] [--iters 10]

Prints the CUDA-event time (median, L2 flushed before each run) and the
expert-GEMM FLOP rate (fwd 2 GEMMs, bwd 4 GEMMs of the routed rows).
"""
from __future__ import annotations

import argparse
import json

import torch

from omnicoder.benchmarks.timing import time_fn
from omnicoder.ops import _ext
from omnicoder.ops.moe import moe_ffn


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--d", type=int, default=2048)
    ap.add_argument("--experts", type=int, default=32)
    ap.add_argument("--ffn", type=int, default=1408)
    ap.add_argument("--topk", type=int, default=4)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--fwd-only", action="store_true")
    args = ap.parse_args()
    dev = torch.device("cuda")
    torch.manual_seed(0)
    T, D, E, F, k = args.tokens, args.d, args.experts, args.ffn, args.topk
    x = (torch.randn(T, D, device=dev) * 0.5).to(torch.bfloat16).requires_grad_(not args.fwd_only)
    router = (torch.randn(E, D, device=dev) * 0.02).to(torch.bfloat16).requires_grad_(not args.fwd_only)
    w13 = (torch.randn(E, 2 * F, D, device=dev) * 0.02).to(torch.bfloat16).requires_grad_(not args.fwd_only)
    w2 = (torch.randn(E, D, F, device=dev) * 0.02).to(torch.bfloat16).requires_grad_(not args.fwd_only)
    cap = int(1.25 * T * k / E + 0.999)
    gy = torch.randn(T, D, device=dev).to(torch.bfloat16)

    def step():
        out, _ = moe_ffn(x, router, w13, w2, k, cap, True)
        if not args.fwd_only:
            torch.autograd.backward(out, gy)
            x.grad = router.grad = w13.grad = w2.grad = None

    ms = time_fn(step, iters=args.iters)
    _ext.check_status()
    rows = T * k
    gemm_flops = 2 * rows * D * 2 * F + 2 * rows * F * D
    flops = gemm_flops * (1 if args.fwd_only else 3)
    res = {"ms": ms, "tokens": T, "d": D, "experts": E, "ffn": F, "topk": k,
           "expert_gemm_tflops": flops / ms / 1e9, "fwd_only": args.fwd_only}
    print(json.dumps(res))


if __name__ == "__main__":
    main()
