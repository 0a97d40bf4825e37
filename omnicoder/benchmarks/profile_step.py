"""Per-kernel time breakdown of one training step (CUDA kernel durations from the
PyTorch profiler; shares are what matters, the bench number comes from bench.py).

    python -m omnicoder.benchmarks.profile_step [--preset moe_mla_24l] [--layers 4] [--seq 4096] [--mb 2]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 \
        -m omnicoder.benchmarks.profile_step ...      # expert x data parallel; rank 0 reports

Kernels on NCCL's streams overlap the compute stream, so their share is an
upper bound of what they cost.
"""
from __future__ import annotations

import argparse
import collections
import datetime
import json
import os
import re

import torch

from omnicoder.config import TrainConfig, get_preset
from omnicoder.models.lm import build_model
from omnicoder.training.engine import Trainer, synthetic_batch


def family(name: str) -> str:
    n = name
    if "gemm_sm100_kernel" in n:
        mode = re.search(r"gemm_sm100_kernel<(\d+), (\w+), (\w+), (\d+), (\d+)(?:, (\w+))?>", n)
        if mode:
            bn, amn, bmn, epi, md, pair = mode.groups()
            kind = {"0": "dense", "1": "grouped_m", "2": "grouped_k", "3": "allgather"}[md]
            pair = " pair" if pair == "true" else ""
            return f"gemm[{kind} a_mn={amn[0]} b_mn={bmn[0]} epi={epi} bn={bn}{pair}]"
        return "gemm"
    for key in ("ep_exchange_layout", "attn_fwd_kernel", "attn_dkdv_kernel", "attn_dq_kernel", "attn_delta_kernel", "rmsnorm_fwd",
                "rmsnorm_bwd", "rope_kernel", "embedding_fwd", "embedding_bwd", "ce_kernel", "adamw_kernel",
                "sq_norm_kernel", "router_topk", "router_bwd", "plan_count", "plan_scan", "plan_assign",
                "moe_gather", "moe_combine_bwd", "moe_combine_kernel", "moe_scatter_add", "ep_dispatch",
                "ep_push", "ep_combine", "ep_owner_bwd", "ep_pad_rows", "ep_barrier", "decode_split",
                "decode_combine", "decode_mla_tc", "decode_gemv", "skinny_gemm", "skinny_finalize", "kv_cache_write",
                "kv_write", "moe_plan", "int4", "nccl"):
        if key in n:
            return key
    return "torch:" + n[:60]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="moe_mla_24l")
    ap.add_argument("--layers", type=int, default=0, help="override layer count (profiling only)")
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--mb", type=int, default=2)
    ap.add_argument("--json", default=None)
    ap.add_argument("--cuda-graph", default="on", choices=["on", "off"])
    args = ap.parse_args()
    cfg = get_preset(args.preset)
    if args.layers:
        cfg.n_layers = args.layers
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    par = None
    if world > 1:
        import torch.distributed as dist

        from omnicoder.parallel.expert_data import ExpertDataParallel
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        par = ExpertDataParallel(dist.group.WORLD,
                                 arena_bytes=ExpertDataParallel.arena_bytes_for(cfg, args.mb * args.seq, world))
    model = build_model(cfg, device=dev, seed=0, ep=par) if par is not None else build_model(cfg, device=dev, seed=0)
    trainer = Trainer(model, TrainConfig(lr=3e-4, warmup_steps=10, max_steps=100, grad_clip=1.0), par,
                      cuda_graph=args.cuda_graph == "on")
    batches = [synthetic_batch(args.mb, args.seq, cfg.vocab_size, rank, i, device=dev) for i in range(4)]
    for b in batches[:3]:
        trainer.step(*b, assume_all_valid=True)
    torch.cuda.synchronize()
    from torch.profiler import ProfilerActivity, profile

    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        trainer.step(*batches[3], assume_all_valid=True)
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    total = 0.0
    for ev in prof.events():
        if ev.device_type is None or not str(ev.device_type).endswith("CUDA"):
            continue
        us = ev.device_time_total if hasattr(ev, "device_time_total") else ev.cuda_time_total
        f = family(ev.name)
        agg[f][0] += 1
        agg[f][1] += us / 1000.0
        total += us / 1000.0
    rows = sorted(agg.items(), key=lambda kv: -kv[1][1])
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
        if rank != 0:
            return
    print(f"{'kernel family':60s} {'count':>6s} {'ms':>9s} {'share':>7s}")
    for name, (cnt, ms) in rows:
        print(f"{name:60s} {cnt:6d} {ms:9.3f} {100 * ms / total:6.1f}%")
    print(f"{'TOTAL':60s} {sum(c for c, _ in agg.values()):6d} {total:9.3f}")
    if args.json:
        with open(args.json, "w") as f:
            json.dump({"layers": cfg.n_layers, "total_ms": total,
                       "rows": [{"name": n, "count": c, "ms": m} for n, (c, m) in rows]}, f, indent=1)


if __name__ == "__main__":
    main()
