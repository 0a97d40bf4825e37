"""Expert-parallel MoE layer microbenchmark (forward + backward): the fused
NVLink peer-memory exchange against the NCCL all_to_all_single + PyTorch
expert-math baseline, on the same routing.

    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \\
        -m omnicoder.benchmarks.bench_ep_moe [--tokens 8192 --dim 4096 --experts 64 --ffn 1408 --topk 6 --cf 1.25]

Per rank: `tokens` bf16 activations ~N(0, 1); router weights scaled so the
router logits are ~N(0, 1); 64 SwiGLU experts (E / N per rank) of ffn 1408
with N(0, 0.02) bf16 weights; top-6 softmax routing, renormalised; expert
capacity = ceil(cf * N * tokens * k / E) over the whole group.  Device-timed
with CUDA events (max over ranks) around forward + backward of one layer;
inputs (>= 67 MB) and expert weights exceed L2 only together, so L2 is
flushed before every timed iteration.

Transports: p2p (fused NVLink exchange, bf16 expert GEMMs whose epilogues store the output rows
into the sources' slots), p2p_gate (the same, with the grouped GEMMs starting each tile as the
sources of its rows signal instead of after a barrier), p2p_ret (local GEMM outputs returned by a copy kernel
after the GEMM), p2p_fp8 (the same
exchange with block-scaled fp8 expert GEMMs -- 1 x 128 activation and 128 x 128
weight scales, power-of-two -- in the forward (SwiGLU and requantisation in the
gate|up epilogue) and in the input gradient through the gate|up experts; the
SwiGLU-backward and weight-gradient GEMMs in bf16), nccl (baseline).

Roofline of the fused path per rank: the slower of (expert GEMM FLOPs of
forward + backward at the measured sustained bf16 peak) and (bytes that must
cross NVLink at 770 GB/s per direction: dispatch rows, combine rows, their
gradients).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics

import torch
import torch.distributed as dist


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--dim", type=int, default=4096)
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--ffn", type=int, default=1408)
    ap.add_argument("--topk", type=int, default=6)
    ap.add_argument("--cf", type=float, default=1.25)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--transports", default="p2p,p2p_gate,p2p_ret,p2p_fp8,nccl",
                    help="p2p (bf16 expert GEMMs), p2p_fp8 (block-scaled fp8 forward expert GEMMs), nccl")
    a = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    from omnicoder.benchmarks.timing import flush_l2
    from omnicoder.ops import _ext
    from omnicoder.parallel.expert import EPContext, ep_moe_ffn

    T, D, E, F, k = a.tokens, a.dim, a.experts, a.ffn, a.topk
    El = E // world
    cap = math.ceil(a.cf * world * T * k / E)
    g = torch.Generator(device="cpu").manual_seed(1000 + rank)
    x = torch.randn(T, D, generator=g).to(dev, torch.bfloat16).requires_grad_(True)
    dy = torch.randn(T, D, generator=g).to(dev, torch.bfloat16)
    gw = torch.Generator(device="cpu").manual_seed(1)
    wr = (torch.randn(E, D, generator=gw) / math.sqrt(D)).to(dev, torch.bfloat16).requires_grad_(True)
    w13 = (torch.randn(El, 2 * F, D, generator=g) * 0.02).to(dev, torch.bfloat16).requires_grad_(True)
    w2 = (torch.randn(El, D, F, generator=g) * 0.02).to(dev, torch.bfloat16).requires_grad_(True)
    rows = int(T * k * a.cf * 1.1) + E * 128
    results = {}
    for tr in a.transports.split(","):
        fp8 = tr == "p2p_fp8"
        ep = EPContext(dist.group.WORLD, transport="nccl" if tr == "nccl" else "p2p", device=dev,
                       arena_bytes=rows * (4 * D * 2 + 16), epilogue_push=tr != "p2p_ret",
                       gate_tiles=tr == "p2p_gate")
        if fp8:
            ep.set_fp8_weights(w13, w2)   # once per optimiser step in training; outside the timed region

        def step():
            ep.begin_step()
            y, _ = ep_moe_ffn(x, wr, w13, w2, k, ep, capacity=cap)
            y.backward(dy)

        for _ in range(a.warmup):
            step()
        torch.cuda.synchronize()
        _ext.check_status()
        times = []
        for _ in range(a.iters):
            flush_l2()
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
        results[tr] = float(t.item())
        del ep
        torch.cuda.empty_cache()
    # roofline of the fused path (per rank)
    kept = min(T * k, cap * E // world)                     # rows processed per rank on average
    flops = 3 * 2 * kept * D * (3 * F)                      # fwd + 2x bwd, gate|up (2F) + down (F)
    remote = (world - 1) / world
    nvl_bytes = 4 * T * k * D * 2 * remote                  # dispatch, combine, and their gradients
    peaks = {"bf16_tflops_sustained": 1366.0}
    try:
        peaks = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..",
                                            "MEASURED_PEAKS.json")))
    except OSError:
        pass
    t_compute = flops / (peaks.get("bf16_tflops_sustained", 1366.0) * 1e12) * 1e3
    t_link = nvl_bytes / 770e9 * 1e3
    roof = max(t_compute, t_link)
    if rank == 0:
        out = {"bench": "expert-parallel MoE layer fwd+bwd", "n_gpus": world, "tokens_per_rank": T, "dim": D,
               "experts": E, "ffn": F, "topk": k, "capacity_factor": a.cf, "capacity": cap,
               "ms": results, "tokens_per_s": {t: world * T / (v / 1e3) for t, v in results.items()},
               "roofline_ms": roof, "roofline_terms_ms": {"compute": t_compute, "nvlink": t_link},
               "fraction_of_roofline": {t: roof / v for t, v in results.items()}}
        if "p2p" in results and "nccl" in results:
            out["speedup_vs_nccl"] = results["nccl"] / results["p2p"]
        print(json.dumps(out), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
