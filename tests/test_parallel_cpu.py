"""Expert parallel x data parallel (ZeRO-1) training step on CPU ranks (gloo):
the loss and the updated parameters of every rank must equal one process
training the same model on the concatenated batch."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig, TrainConfig


def _cfg(capacity_factor: float) -> ModelConfig:
    return ModelConfig(name="ep_test", vocab_size=512, d_model=64, n_layers=2, n_heads=4, ffn_dim=128,
                       tie_embeddings=False, max_seq_len=64, attn=AttentionConfig(kind="mha"),
                       moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=64, n_shared_experts=1,
                                     capacity_factor=capacity_factor, aux_loss_alpha=0.0))


def _tcfg():
    # eps large enough that Adam's first step is not dominated by the sign of ~1e-9 gradients
    return TrainConfig(lr=1e-3, warmup_steps=0, max_steps=10, grad_clip=1.0, weight_decay=0.1, eps=1e-6,
                       betas=(0.9, 0.95))


def _batch(world, seq=32):
    g = torch.Generator().manual_seed(123)
    ids = torch.randint(0, 512, (2 * world, seq), generator=g)
    lab = torch.randint(0, 512, (2 * world, seq), generator=g)
    return ids, lab


def _worker(rank, world, port, cf, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from omnicoder.models.lm import build_model
        from omnicoder.parallel.expert_data import ExpertDataParallel
        from omnicoder.training.engine import Trainer

        cfg = _cfg(cf)
        ids, lab = _batch(world)
        # single-process reference on the whole batch
        ref = build_model(cfg, device="cpu", seed=0)
        rt = Trainer(ref, _tcfg())
        ref_stats = [float(rt.step(ids, lab).loss) for _ in range(2)]
        # expert x data parallel over `world` ranks
        par = ExpertDataParallel(dist.group.WORLD)
        model = build_model(cfg, device="cpu", seed=0, ep=par)
        tr = Trainer(model, _tcfg(), par)
        mine = ids.chunk(world)[rank], lab.chunk(world)[rank]
        stats = []
        for _ in range(2):
            loss = tr.step(*mine).loss.detach()
            dist.all_reduce(loss)
            stats.append(float(loss) / world)
        lo, hi = par.expert_slice(cfg.moe.n_experts)
        ref_sd = ref.state_dict()
        worst = 0.0
        for name, p in model.state_dict().items():
            r = ref_sd[name]
            if name.endswith("ffn.w13") or name.endswith("ffn.w2"):
                r = r[lo:hi]
            worst = max(worst, float((p - r).abs().max()))
        q.put((rank, ref_stats, stats, worst))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("cf,world", [(0.0, 2), (1.0, 2), (0.0, 4)])
def test_ep_dp_zero1_matches_single_process(cf, world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cf, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ref_stats, stats, worst in res:
        for a, b in zip(ref_stats, stats):
            assert abs(a - b) < 1e-4, (rank, ref_stats, stats)
        assert worst < 1e-4, (rank, worst)
