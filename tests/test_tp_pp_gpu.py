"""Tensor parallel (+ sequence parallel) and 1F1B pipeline training on 2 GPUs, and a
4-stage pipeline on 4 (one process per GPU): the group-mean loss of three steps must track one GPU
training the same model on the same batch (bf16 tolerance).  Tensor parallel
runs with NCCL collectives and with the fused peer-memory collectives
(all-gather inside the consuming GEMM's loads, reduce-scatter in the producing
GEMM's epilogue)."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg():
    from omnicoder.config import AttentionConfig, ModelConfig
    return ModelConfig(name="tpp", vocab_size=4096, d_model=512, n_layers=4, n_heads=8, ffn_dim=1024,
                       tie_embeddings=False, max_seq_len=512, attn=AttentionConfig(kind="gqa", n_kv_heads=2))


def _worker(rank, world, port, mode, q):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from omnicoder.config import TrainConfig
        from omnicoder.models.lm import build_model
        from omnicoder.ops import _ext
        from omnicoder.training.engine import Trainer, synthetic_batch
        tc = TrainConfig(lr=1e-3, warmup_steps=0, max_steps=10, grad_clip=1.0)
        ids, lab = synthetic_batch(4, 256, 4096, seed=1, step=0, device=dev)
        ref = build_model(_cfg(), device=dev, seed=0)
        rt = Trainer(ref, tc)
        ref_l = [float(rt.step(ids, lab).loss) for _ in range(3)]
        del rt, ref
        if mode in ("tp", "tp_p2p"):
            from omnicoder.parallel.tensor import TensorParallel
            par = TensorParallel(dist.group.WORLD, transport="p2p" if mode == "tp_p2p" else "nccl")
            m = build_model(_cfg(), device=dev, seed=0, tp=par)
            tr = Trainer(m, tc, par)
            got = []
            for _ in range(3):
                l = tr.step(ids, lab).loss.detach().float()
                dist.all_reduce(l)
                got.append(float(l) / world)
        else:
            from omnicoder.parallel.pipeline import PipelineTrainer
            m = build_model(_cfg(), device=dev, seed=0)
            pt = PipelineTrainer(m, tc, n_micro=2 if world == 2 else 4)
            got = [float(pt.step(ids, lab)) for _ in range(3)]
        torch.cuda.synchronize()
        C = _ext.load()
        code = C.status()[0]
        C.status_reset()
        q.put((rank, {"ref": ref_l, "got": got, "status": code}))
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _run(mode, world=2):
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, v = q.get(timeout=600)
            res[r] = v
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


@pytest.mark.parametrize("mode,world", [("tp", 2), ("tp_p2p", 2), ("pp", 2), ("pp", 4)])
def test_tp_and_pp_track_single_gpu(mode, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    for rank, out in _run(mode, world).items():
        assert isinstance(out, dict), out
        assert out["status"] == 0
        for a, b in zip(out["ref"], out["got"]):
            assert abs(a - b) < 2e-2 * max(1.0, abs(a)), (mode, out)
