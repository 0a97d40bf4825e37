"""Tensor-parallel (sequence-parallel) SwiGLU MLP block, forward + backward: the
fused peer-memory collectives (each peer's token shard copied once over
NVLink while the gate|up GEMM already runs on the shards present; the down
GEMM's epilogue stores its partial tiles into the row owners' staging slots) against NCCL all_gather /
reduce_scatter around the same GEMMs.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m omnicoder.benchmarks.bench_tp [--tokens 8192 --dim 6144 --ffn 16384]

Shapes: the dense 20B configuration (d_model 6144, SwiGLU ffn 16384), one
8192-token sequence per tensor-parallel group (tokens / N per rank between
blocks).  Device-timed (CUDA events, median of `iters`, max over ranks).
Roofline of the fused block per rank: the slower of the GEMM FLOPs of forward +
backward at the measured sustained bf16 rate and the bytes the collectives move
over NVLink (4 all-gathers / reduce-scatters of tokens x d_model bf16, each
(N-1)/N remote) at 770 GB/s.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics

import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--dim", type=int, default=6144)
    ap.add_argument("--ffn", type=int, default=16384)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    a = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    from omnicoder.ops import _ext
    from omnicoder.parallel.tensor import TPContext, tp_swiglu_mlp

    T, D, F = a.tokens, a.dim, a.ffn
    rows = T // world
    Fl = F // world
    g = torch.Generator(device="cpu").manual_seed(100 + rank)
    x = torch.randn(rows, D, generator=g).to(dev, torch.bfloat16).requires_grad_(True)
    dy = torch.randn(rows, D, generator=g).to(dev, torch.bfloat16)
    w13 = (torch.randn(2 * Fl, D, generator=g) * 0.02).to(dev, torch.bfloat16).requires_grad_(True)
    w2 = (torch.randn(D, Fl, generator=g) * 0.02).to(dev, torch.bfloat16).requires_grad_(True)
    res = {}
    for tr in ("p2p", "nccl"):
        tp = TPContext(dist.group.WORLD, transport=tr, arena_bytes=2 * world * rows * max(D, 2 * Fl) * 2)

        def step():
            if tr == "p2p":
                y = tp_swiglu_mlp(x, w13, w2, tp, residual=x)
            else:
                from omnicoder.ops.layers import swiglu_mlp
                from omnicoder.parallel.tensor import all_gather_seq, reduce_scatter_seq
                y = reduce_scatter_seq(swiglu_mlp(all_gather_seq(x, tp), w13, w2), tp) + x
            y.backward(dy)

        for _ in range(a.warmup):
            step()
        torch.cuda.synchronize()
        _ext.check_status()
        times = []
        for _ in range(a.iters):
            dist.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            step()
            e1.record()
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        _ext.check_status()
        t = torch.tensor([statistics.median(times)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[tr] = float(t.item())
    flops = 3 * (2 * T * D * 2 * Fl + 2 * T * Fl * D)       # fwd + bwd of gate|up and down
    nvl = 4 * T * D * 2 * (world - 1) / world
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..",
                                            "MEASURED_PEAKS.json")))
    except OSError:
        pass
    t_c = flops / (peaks.get("bf16_tflops_sustained", 1366.0) * 1e12) * 1e3
    t_l = nvl / 770e9 * 1e3
    roof = max(t_c, t_l)
    if rank == 0:
        print(json.dumps({"bench": "tensor-parallel SwiGLU MLP fwd+bwd", "n_gpus": world, "tokens": T, "dim": D,
                          "ffn": F, "ms": res, "speedup_vs_nccl": res["nccl"] / res["p2p"], "roofline_ms": roof,
                          "roofline_terms_ms": {"compute": t_c, "nvlink": t_l},
                          "fraction_of_roofline": {k: roof / v for k, v in res.items()}}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
