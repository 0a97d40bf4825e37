"""Dense 20B training step with tensor parallelism + sequence parallelism over all ranks.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        -m omnicoder.benchmarks.bench_dense_tp [--global-batch 64] [--steps 2 --warmup 1] \\
        [--transport nccl|p2p] [--arms ours,baseline] [--layers 48] [--pp P] [--fp8]

Model: dense_20b (48 layers, d_model 6144, 48 query / 8 KV heads of 128, SwiGLU 16384,
vocab 32000), sequence 8192, random N(0, 0.02) weights, uniform random token ids; bf16
compute with fp32 master weights and AdamW state.  Every rank of the tensor-parallel group
sees the same sequences; the global batch is processed one sequence at a time with
gradient accumulation and one optimiser step.

Arms (same data, same step):
  ours      this package's model and kernels under omnicoder.parallel.tensor.TensorParallel
            (transport "nccl": all-gather / reduce-scatter around this package's GEMMs and
            flash attention; "p2p": the fused peer-memory all-gather -> GEMM and GEMM ->
            reduce-scatter collectives);
  baseline  plain PyTorch + NCCL + cuBLAS (omnicoder.baselines.torch_tp).
`--fp8`: the block projections' forward and input-gradient GEMMs in fp8 -- ours with
1 x 128 / 128 x 128 block scales (power-of-two, applied by the tensor core), the baseline
with row-wise scales through torch._scaled_mm; weight gradients bf16 in both.
`--pp P` runs the second layout instead: P pipeline stages (1F1B over NCCL point-to-point,
omnicoder.parallel.pipeline) x tensor parallel N / P inside each stage (rank = stage x TP +
tp rank), the global batch split into micro-batches of one sequence; only this package's arm.
Device time with CUDA events, max over ranks; tokens/s = global batch x 8192 / step time.
"""
from __future__ import annotations

import argparse
import datetime
import gc
import json
import os

import torch
import torch.distributed as dist


def _time(step, ids, lab, warmup, steps, dev):
    for _ in range(warmup):
        step(ids, lab)
    torch.cuda.synchronize()
    dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    loss = None
    for _ in range(steps):
        loss = step(ids, lab)
    e1.record()
    torch.cuda.synchronize()
    t = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()), float(loss)


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--global-batch", type=int, default=64)
    ap.add_argument("--seq", type=int, default=8192)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--layers", type=int, default=0, help="override the layer count (quick runs)")
    ap.add_argument("--transport", default="nccl", choices=["nccl", "p2p"])
    ap.add_argument("--arms", default="ours,baseline")
    ap.add_argument("--json", default=None)
    ap.add_argument("--pp", type=int, default=1, help="pipeline stages (tensor parallel = N / pp inside each)")
    ap.add_argument("--fp8", action="store_true", help="block-scaled fp8 projections (forward and dgrad GEMMs)")
    a = ap.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
    from omnicoder.config import TrainConfig, get_preset
    from omnicoder.training.engine import synthetic_batch
    from omnicoder.utils.flops import train_flops_per_token

    cfg = get_preset("dense_20b")
    cfg.max_seq_len = max(cfg.max_seq_len, a.seq)
    if a.layers:
        cfg.n_layers = a.layers
    G, S = a.global_batch, a.seq
    tcfg = TrainConfig(lr=3e-4, warmup_steps=10, max_steps=1000, micro_batch=1, seq_len=S, grad_accum=G,
                       grad_clip=1.0, weight_decay=0.1, betas=(0.9, 0.95))
    ids, lab = synthetic_batch(G, S, cfg.vocab_size, seed=0, step=0, device=dev)   # same data on every rank
    res = {}
    if a.pp > 1:
        from omnicoder.models.lm import build_model
        from omnicoder.parallel.pipeline import PipelineTrainer
        from omnicoder.parallel.tensor import TensorParallel
        T = world // a.pp
        if T * a.pp != world:
            raise SystemExit(f"{world} ranks do not split into {a.pp} stages")
        tp_groups = [dist.new_group(list(range(s_ * T, (s_ + 1) * T))) for s_ in range(a.pp)]
        pp_groups = [dist.new_group(list(range(t_, world, T))) for t_ in range(T)]
        stage, t = rank // T, rank % T
        par = TensorParallel(tp_groups[stage], transport=a.transport, fp8=a.fp8) if T > 1 else None
        model = build_model(cfg, device=dev, seed=1234, tp=par)
        pt = PipelineTrainer(model, tcfg, group=pp_groups[t], n_micro=G, tp=par)
        del model
        gc.collect()
        torch.cuda.empty_cache()
        ms, loss = _time(pt.step, ids, lab, a.warmup, a.steps, dev)
        res["ours"] = {"ms_per_step": ms, "tokens_per_s": G * S / (ms / 1e3), "loss": loss,
                       "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 1e9}
        a.arms = ""
    for arm in [x for x in a.arms.split(",") if x]:
        if arm == "ours":
            from omnicoder.models.lm import build_model
            from omnicoder.parallel.tensor import TensorParallel
            from omnicoder.training.engine import Trainer
            par = TensorParallel(dist.group.WORLD, transport=a.transport, fp8=a.fp8)
            model = build_model(cfg, device=dev, seed=1234, tp=par)
            tr = Trainer(model, tcfg, par)
            step = lambda i, l: tr.step(i, l, assume_all_valid=True).loss
        elif arm == "baseline":
            from omnicoder.baselines.torch_tp import TorchDenseTPLM, TorchTPTrainer
            model = TorchDenseTPLM(cfg, dev, dist.group.WORLD, seed=1234, fp8=a.fp8)
            tr = TorchTPTrainer(model, tcfg)
            step = tr.step
        else:
            raise SystemExit(f"unknown arm {arm!r}")
        ms, loss = _time(step, ids, lab, a.warmup, a.steps, dev)
        res[arm] = {"ms_per_step": ms, "tokens_per_s": G * S / (ms / 1e3), "loss": loss,
                    "peak_mem_gb": torch.cuda.max_memory_allocated(dev) / 1e9}
        del step, tr, model
        gc.collect()
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(dev)
    fpt = train_flops_per_token(cfg, S)
    for r in res.values():
        r["model_tflops_per_gpu"] = r["tokens_per_s"] * fpt / world / 1e12
    if rank == 0:
        out = {"bench": "dense 20B training step, tensor + sequence parallel", "n_gpus": world,
               "parallelism": (f"pp{a.pp}xtp{world // a.pp}+sp" if a.pp > 1 else f"tp{world}+sp"),
               "transport": a.transport, "model": f"{cfg.name} {cfg.n_layers}L",
               "global_batch": G, "seq_len": S,
               "dtype": ("fp8 e4m3 projections (fprop + dgrad), bf16 elsewhere" if a.fp8 else "bf16")
               + " (fp32 master weights, AdamW)",
               "data": "synthetic (uniform random token ids, random-init N(0,0.02))",
               "train_gflop_per_token": fpt / 1e9, "arms": res}
        if "ours" in res and "baseline" in res:
            out["vs_baseline"] = res["ours"]["tokens_per_s"] / res["baseline"]["tokens_per_s"]
        print(json.dumps(out), flush=True)
        if a.json:
            with open(a.json, "w") as f:
                json.dump(out, f, indent=1)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
