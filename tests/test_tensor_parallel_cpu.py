"""Tensor parallel + sequence parallel training step on CPU ranks (gloo): the
group-mean loss and every parameter after two optimiser steps (sharded ones
against the matching slice) must equal one process on the same batch."""
import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from omnicoder.config import AttentionConfig, ModelConfig, TrainConfig


def _cfg():
    return ModelConfig(name="tp_test", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128,
                       tie_embeddings=False, max_seq_len=64, attn=AttentionConfig(kind="gqa", n_kv_heads=2))


def _tc():
    return TrainConfig(lr=1e-3, warmup_steps=0, max_steps=10, grad_clip=0.5, weight_decay=0.1, eps=1e-6,
                       betas=(0.9, 0.95))


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from omnicoder.models.lm import build_model
        from omnicoder.parallel.tensor import TensorParallel
        from omnicoder.training.engine import Trainer

        g = torch.Generator().manual_seed(5)
        ids = torch.randint(0, 300, (2, 32), generator=g)
        lab = torch.randint(0, 300, (2, 32), generator=g)
        ref = build_model(_cfg(), device="cpu", seed=0)
        rt = Trainer(ref, _tc())
        ref_losses = [float(rt.step(ids, lab).loss) for _ in range(2)]
        par = TensorParallel(dist.group.WORLD)
        m = build_model(_cfg(), device="cpu", seed=0, tp=par)
        tr = Trainer(m, _tc(), par)
        losses = []
        for _ in range(2):
            l = tr.step(ids, lab).loss.detach().clone()
            dist.all_reduce(l)
            losses.append(float(l) / world)
        worst = 0.0
        rsd = ref.state_dict()
        H, Hk, hd, D, F = 4, 2, 16, 64, 128
        for name, p in m.state_dict().items():
            r = rsd[name]
            if name.endswith("attn.wqkv"):
                h0, h1 = rank * H // world, (rank + 1) * H // world
                k0, k1 = rank * Hk // world, (rank + 1) * Hk // world
                r = torch.cat([r[h0 * hd:h1 * hd], r[(H + k0) * hd:(H + k1) * hd], r[(H + Hk + k0) * hd:(H + Hk + k1) * hd]])
            elif name.endswith("attn.wo"):
                r = r[:, rank * H // world * hd:(rank + 1) * H // world * hd]
            elif name.endswith("ffn.w13"):
                r = r[rank * 2 * F // world:(rank + 1) * 2 * F // world]
            elif name.endswith("ffn.w2"):
                r = r[:, rank * F // world:(rank + 1) * F // world]
            worst = max(worst, float((p - r).abs().max()))
        q.put((rank, ref_losses, losses, worst))
    finally:
        dist.destroy_process_group()


def test_tp_sp_matches_single_process():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ref, got, worst in res:
        for a, b in zip(ref, got):
            assert abs(a - b) < 1e-4, (rank, ref, got)
        assert worst < 1e-4, (rank, worst)


def _cfg8():
    return ModelConfig(name="tp_fp8_test", vocab_size=300, d_model=128, n_layers=2, n_heads=4, ffn_dim=256,
                       tie_embeddings=False, max_seq_len=64,
                       attn=AttentionConfig(kind="gqa", n_kv_heads=2, head_dim=64))


def _worker_fp8(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from omnicoder.models.lm import build_model
        from omnicoder.parallel.tensor import TensorParallel
        from omnicoder.training.engine import Trainer

        g = torch.Generator().manual_seed(5)
        ids = torch.randint(0, 300, (2, 32), generator=g)
        lab = torch.randint(0, 300, (2, 32), generator=g)
        ref = build_model(_cfg8(), device="cpu", seed=0)
        ref_losses = [float(Trainer(ref, _tc()).step(ids, lab).loss)]
        par = TensorParallel(dist.group.WORLD, fp8=True)
        m = build_model(_cfg8(), device="cpu", seed=0, tp=par)
        tr = Trainer(m, _tc(), par)
        losses = []
        for _ in range(3):
            l = tr.step(ids, lab).loss.detach().clone()
            dist.all_reduce(l)
            losses.append(float(l) / world)
        q.put((rank, ref_losses, losses))
    finally:
        dist.destroy_process_group()


def test_tp_fp8_projections_track_full_precision():
    """fp8 block-scaled projections under TP=2: the first loss equals the full-precision
    single-process loss within the fp8 quantisation error, and training lowers it."""
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker_fp8, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ref, got in res:
        assert abs(ref[0] - got[0]) / ref[0] < 5e-3, (rank, ref, got)
        assert got[-1] < got[0], got
