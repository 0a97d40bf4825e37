"""1F1B pipeline over 2 and 4 CPU stages, and 2 stages x tensor parallel 2 (gloo point-to-point):
the loss and the updated parameters of each stage must equal one process on the same batch."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from omnicoder.config import AttentionConfig, ModelConfig, TrainConfig


def _cfg():
    return ModelConfig(name="pp_test", vocab_size=300, d_model=64, n_layers=4, n_heads=4, ffn_dim=128,
                       tie_embeddings=False, max_seq_len=64, attn=AttentionConfig(kind="gqa", n_kv_heads=2))


def _tc():
    return TrainConfig(lr=1e-3, warmup_steps=0, max_steps=10, grad_clip=0.5, weight_decay=0.1, eps=1e-6,
                       betas=(0.9, 0.95))


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from omnicoder.models.lm import build_model
        from omnicoder.parallel.pipeline import PipelineTrainer
        from omnicoder.training.engine import Trainer

        g = torch.Generator().manual_seed(9)
        ids = torch.randint(0, 300, (8, 16), generator=g)
        lab = torch.randint(0, 300, (8, 16), generator=g)
        ref = build_model(_cfg(), device="cpu", seed=0)
        rt = Trainer(ref, _tc())
        ref_losses = [float(rt.step(ids, lab).loss) for _ in range(2)]
        m = build_model(_cfg(), device="cpu", seed=0)
        pt = PipelineTrainer(m, _tc(), n_micro=4)
        losses = [float(pt.step(ids, lab)) for _ in range(2)]
        rsd = ref.state_dict()
        names = {id(p): n for n, p in m.named_parameters()}
        worst = max(float((p - rsd[names[id(p)]]).abs().max()) for p in pt.stage.parameters())
        q.put((rank, ref_losses, losses, worst))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("stages", [2, 4])
def test_pipeline_1f1b_matches_single_process(stages):
    """2 and 4 stages (4: warm-up, steady state with paired exchanges and cool-down all non-trivial)."""
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, stages, port, q)) for r in range(stages)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(stages)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ref, got, worst in res:
        for a, b in zip(ref, got):
            assert abs(a - b) < 1e-4, (rank, ref, got)
        assert worst < 1e-4, (rank, worst)


def _pptp_worker(rank, world, port, q):
    """2 pipeline stages x tensor parallel 2 (rank = stage * 2 + tp rank)."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from omnicoder.models.lm import build_model
        from omnicoder.parallel.pipeline import PipelineTrainer
        from omnicoder.parallel.tensor import TensorParallel
        from omnicoder.training.engine import Trainer

        tp_groups = [dist.new_group([0, 1]), dist.new_group([2, 3])]
        pp_groups = [dist.new_group([0, 2]), dist.new_group([1, 3])]
        stage, t = rank // 2, rank % 2
        g = torch.Generator().manual_seed(9)
        ids = torch.randint(0, 300, (8, 16), generator=g)
        lab = torch.randint(0, 300, (8, 16), generator=g)
        ref = build_model(_cfg(), device="cpu", seed=0)
        rt = Trainer(ref, _tc())
        ref_losses = [float(rt.step(ids, lab).loss) for _ in range(3)]
        tp = TensorParallel(tp_groups[stage])
        m = build_model(_cfg(), device="cpu", seed=0, tp=tp)
        pt = PipelineTrainer(m, _tc(), group=pp_groups[t], n_micro=4, tp=tp)
        losses = [float(pt.step(ids, lab)) for _ in range(3)]
        rsd = ref.state_dict()
        names = {id(p): n for n, p in m.named_parameters()}
        worst = max(float((p - rsd[names[id(p)]]).abs().max()) for p in pt.stage.parameters()
                    if not getattr(p, "tp_sharded", False))
        q.put((rank, ref_losses, losses, worst))
    finally:
        dist.destroy_process_group()


def test_pipeline_with_tensor_parallel_stages_matches_single_process():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_pptp_worker, args=(r, 4, port, q)) for r in range(4)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(4)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ref, got, worst in res:
        for a, b in zip(ref, got):
            assert abs(a - b) < 1e-4, (rank, ref, got)
        assert worst < 1e-4, (rank, worst)
