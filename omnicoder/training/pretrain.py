"""LM pretraining entry point: ``python -m omnicoder.training.pretrain``.

Same entry point and main flags as the reference trainer
(src/omnicoder/training/pretrain.py:31-1157: --data --batch_size --seq_len
--steps --lr --device --out --resume_ckpt --state_out --grad_accum
--mobile_preset --log_interval --log_file --save_interval --rope_scale
--rope_base --target_ctx --aux_lb_coef --aux_zloss_coef).  Differences:

* the model is the spec family (omnicoder.models.lm) built from a named preset
  (`--preset`, or the reference's `--mobile_preset` names);
* launched under torchrun (WORLD_SIZE > 1) it trains expert parallel x data
  parallel with ZeRO-1 (omnicoder.parallel.expert_data); every rank reads a
  disjoint subset of the corpus;
* `--data synthetic` trains on uniform random ids (the benchmark workload);
* the optimiser state really is restored on resume (the reference re-creates
  its optimiser after loading it, pretrain.py:582);
* throughput is logged from CUDA events (device time), not host wall clock.

Checkpoints: `--out` gets the model (rank 0 gathers the expert shards into one
consolidated state_dict, with SwiGLU w1/w3 split); `--state_out` gets the
trainer step and optimiser state (one shard file per rank under EP/ZeRO).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import time

import torch
import torch.distributed as dist

from ..config import TrainConfig, get_preset, get_rope_scale_for_target_ctx
from ..models.lm import MoEFFN, build_model
from .checkpoint import _atomic_save, maybe_load_checkpoint
from .data import JsonlTextDataset, SyntheticTokens, TextFolderDataset, batches
from .engine import Trainer


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description="omnicoder LM pretraining")
    ap.add_argument("--data", default=os.getenv("OMNICODER_PRETRAIN_DATA", "synthetic"),
                    help="folder of text files, a .jsonl file, or 'synthetic'")
    ap.add_argument("--batch_size", type=int, default=4, help="sequences per rank per step")
    ap.add_argument("--seq_len", type=int, default=256)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--lr", type=float, default=3e-4)
    ap.add_argument("--warmup", type=int, default=0)
    ap.add_argument("--weight_decay", type=float, default=0.1)
    ap.add_argument("--grad_clip", type=float, default=1.0)
    ap.add_argument("--grad_accum", type=int, default=1)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--preset", default=None, help="model preset (tiny_moe, moe_mla_24l, dense_20b, ...)")
    ap.add_argument("--mobile_preset", default=os.getenv("OMNICODER_STUDENT_PRESET", "tiny_moe"))
    ap.add_argument("--out", default="weights/omnicoder.pt")
    ap.add_argument("--resume_ckpt", default="")
    ap.add_argument("--state_out", default="weights/pretrain_state.pt")
    ap.add_argument("--log_interval", type=int, default=10)
    ap.add_argument("--log_file", default="weights/pretrain_log.jsonl")
    ap.add_argument("--save_interval", type=int, default=0)
    ap.add_argument("--rope_scale", type=float, default=1.0)
    ap.add_argument("--rope_base", type=float, default=10000.0)
    ap.add_argument("--target_ctx", type=int, default=0)
    ap.add_argument("--aux_lb_coef", type=float, default=None, help="load-balance loss weight")
    ap.add_argument("--aux_zloss_coef", type=float, default=None, help="router z-loss weight")
    ap.add_argument("--capacity_factor", type=float, default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--tokenizer", default=None, help="local Hugging Face tokenizer directory (default: bytes)")
    ap.add_argument("--ep_transport", default="auto", choices=["auto", "p2p", "nccl"])
    ap.add_argument("--pg_timeout", type=float, default=600.0, help="process-group timeout (s)")
    ap.add_argument("--log_expert_load", action="store_true",
                    help="single process: add per-layer expert load (CV, busiest share) to each log record "
                         "(one extra no-grad forward per log interval)")
    ap.add_argument("--heartbeat_timeout", type=float, default=0.0,
                    help="multi-rank: check every rank's heartbeat before each step, naming a rank that left, "
                         "died or stalled for this many seconds (0: off)")
    return ap.parse_args(argv)


def consolidated_state_dict(model, world: int, group=None) -> dict:
    """Full state_dict with every rank's expert shard gathered (collective; the result is
    only meaningful on rank 0)."""
    sd = {}
    for name, p in model.state_dict().items():
        sd[name] = p.detach()
    if world > 1:
        for mname, m in model.named_modules():
            if isinstance(m, MoEFFN) and m.ep is not None:
                for pn in ("w13", "w2"):
                    t = getattr(m, pn).detach().contiguous()
                    parts = [torch.empty_like(t) for _ in range(world)]
                    dist.all_gather(parts, t, group=group)
                    sd[f"{mname}.{pn}"] = torch.cat(parts, 0)
    return sd


def main(argv=None):
    a = parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device(a.device)
    if dev.type == "cuda":
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
    par = None
    cfg = get_preset(a.preset or a.mobile_preset)
    cfg.max_seq_len = max(cfg.max_seq_len, a.seq_len)
    cfg.attn.rope_theta = a.rope_base
    cfg.attn.rope_scale = get_rope_scale_for_target_ctx(cfg.max_seq_len, a.target_ctx) if a.target_ctx else a.rope_scale
    if a.aux_lb_coef is not None:
        cfg.moe.aux_loss_alpha = a.aux_lb_coef
    if a.aux_zloss_coef is not None:
        cfg.moe.z_loss_beta = a.aux_zloss_coef
    if a.capacity_factor is not None:
        cfg.moe.capacity_factor = a.capacity_factor
    if world > 1:
        dist.init_process_group("nccl" if dev.type == "cuda" else "gloo", timeout=datetime.timedelta(seconds=a.pg_timeout),
                                device_id=dev if dev.type == "cuda" else None)
        from ..parallel.expert_data import ExpertDataParallel
        par = ExpertDataParallel(dist.group.WORLD, transport=a.ep_transport)
    tc = TrainConfig(lr=a.lr, warmup_steps=a.warmup, max_steps=a.steps, grad_clip=a.grad_clip,
                     weight_decay=a.weight_decay, micro_batch=a.batch_size, seq_len=a.seq_len, grad_accum=a.grad_accum,
                     seed=a.seed)
    model = build_model(cfg, device=dev, seed=a.seed, ep=par)
    start = 0
    if a.resume_ckpt:
        rep = maybe_load_checkpoint(model, a.resume_ckpt)
        if rank == 0:
            print(f"[pretrain] resumed model from {a.resume_ckpt}: {rep}", flush=True)
    trainer = Trainer(model, tc, par)
    state_path = a.state_out if world == 1 else f"{a.state_out}.rank{rank}"
    if a.resume_ckpt and os.path.exists(state_path):
        trainer.load_state_dict(torch.load(state_path, map_location="cpu", weights_only=False))
        start = trainer.step_idx
    if a.data == "synthetic":
        src = SyntheticTokens(cfg.vocab_size, a.seq_len, seed=a.seed, rank=rank)
    else:
        from .tokenizer import get_tokenizer
        tok = get_tokenizer(cfg.vocab_size, a.tokenizer)
        src = (JsonlTextDataset(a.data, a.seq_len, tok, rank=rank, world=world) if a.data.endswith(".jsonl")
               else TextFolderDataset(a.data, a.seq_len, tok, rank=rank, world=world))
    it = batches(src, a.batch_size, shuffle_seed=a.seed + start)
    log = open(a.log_file, "a") if (rank == 0 and a.log_file) else None
    if log is not None:
        os.makedirs(os.path.dirname(os.path.abspath(a.log_file)) or ".", exist_ok=True)
    ev0 = torch.cuda.Event(enable_timing=True) if dev.type == "cuda" else None
    ev1 = torch.cuda.Event(enable_timing=True) if dev.type == "cuda" else None
    if ev0 is not None:
        ev0.record()
    from ..parallel.health import FaultInjector, Heartbeat
    hb = Heartbeat(timeout=a.heartbeat_timeout).start() if (world > 1 and a.heartbeat_timeout > 0) else None
    inj = FaultInjector.from_env(device_type=dev.type, world=world)
    try:
        _train_loop(a, trainer, model, it, dev, world, rank, start, state_path, log, ev0, ev1, hb, inj)
    except Exception as e:
        if hb is not None:
            hb.leave(f"{type(e).__name__}: {e}")
        raise
    if hb is not None:
        hb.stop()
    _save(model, trainer, a, world, rank, state_path, a.steps)
    if log is not None:
        log.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _train_loop(a, trainer, model, it, dev, world, rank, start, state_path, log, ev0, ev1, hb, inj):
    from ..utils.flops import train_flops_per_token
    t_last, tok_acc = time.time(), 0
    for step in range(start, a.steps):
        inj.at_step(rank, step, hb)
        if hb is not None:
            hb.check(step)
        ids, lab = next(it)
        st = trainer.step(ids.to(dev, non_blocking=True), lab.to(dev, non_blocking=True))
        tok_acc += ids.numel() * world
        if (step + 1) % a.log_interval == 0 or step + 1 == a.steps:
            loss = float(st.loss)
            if world > 1:
                t = torch.tensor([loss], device=dev)
                dist.all_reduce(t)
                loss = float(t) / world
            if ev1 is not None:
                ev1.record()
                ev1.synchronize()
                secs = ev0.elapsed_time(ev1) / 1000.0
                ev0.record()
            else:
                secs = time.time() - t_last
                t_last = time.time()
            tps = tok_acc / max(secs, 1e-9)
            rec = {"step": step + 1, "loss": loss, "ce": float(st.ce), "aux": float(st.aux), "lr": st.lr,
                   "tokens_per_s": tps, "model_tflops_per_gpu": tps * train_flops_per_token(model.cfg, a.seq_len)
                   / world / 1e12, "time": time.time()}
            if a.log_expert_load and world == 1:
                from ..utils.diagnostics import expert_load
                el = expert_load(model, ids.to(dev))
                rec["expert_load_cv"], rec["expert_max_share"] = el["cv"], el["max_share"]
            tok_acc = 0
            if rank == 0:
                print(f"[pretrain] step {step + 1}/{a.steps} loss {loss:.4f} lr {st.lr:.2e} "
                      f"{rec['tokens_per_s']:.0f} tok/s", flush=True)
                if log is not None:
                    log.write(json.dumps(rec) + "\n")
                    log.flush()
        if a.save_interval and (step + 1) % a.save_interval == 0:
            _save(model, trainer, a, world, rank, state_path, step + 1)


def _save(model, trainer, a, world, rank, state_path, step):
    sd = consolidated_state_dict(model, world)
    if rank == 0 and a.out:
        from ..ops.gemm import split_gate_up
        exp = {}
        for k, v in sd.items():
            if k.endswith(".w13"):
                w1, w3 = split_gate_up(v)
                exp[k[:-4] + ".w1"], exp[k[:-4] + ".w3"] = w1.cpu(), w3.cpu()
            else:
                exp[k] = v.cpu()
        _atomic_save({"model": exp, "config": model.cfg.to_dict(), "step": step}, a.out)
    if a.state_out:
        _atomic_save(trainer.state_dict(), state_path)


if __name__ == "__main__":
    main()
