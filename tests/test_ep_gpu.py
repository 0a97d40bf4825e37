"""Expert-parallel MoE layer over NVLink peer memory on 2 GPUs (one process per
GPU, NCCL for the plumbing): output, input gradient, router gradient and the
local experts' weight gradients of the fused p2p kernels must match the
single-GPU fused MoE layer on the concatenated tokens; the all_to_all (NCCL)
transport must agree as well.  A full expert x data parallel training step must
give the same loss as one GPU on the whole batch.

Runs as child processes with NVLS off; every device wait in the kernels is
bounded and a timeout shows up in the device status word checked here."""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    return err / ref < tol, err / ref


def _layer_worker(rank, world, port, q):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    out = {}
    try:
        from omnicoder.ops import _ext, moe_ffn
        from omnicoder.parallel.expert import EPContext, ep_moe_ffn

        C = _ext.load()
        T, D, E, F, K = 1024, 512, 8, 256, 2
        g = torch.Generator(device="cpu").manual_seed(7)
        xs = (torch.randn(world * T, D, generator=g) * 0.5).to(dev, torch.bfloat16)
        wr = (torch.randn(E, D, generator=g) * 0.05).to(dev, torch.bfloat16)
        w13 = (torch.randn(E, 2 * F, D, generator=g) * 0.05).to(dev, torch.bfloat16)
        w2 = (torch.randn(E, D, F, generator=g) * 0.05).to(dev, torch.bfloat16)
        dys = (torch.randn(world * T, D, generator=g) * 0.1).to(dev, torch.bfloat16)
        El = E // world
        lo, hi = rank * El, (rank + 1) * El
        # (capacity passed to the layer, capacity of the single-GPU reference, variants):
        # variant = (name, transport, layout, buffer factor); the device layout with buffer
        # factor 0.5 bounds every expert at 256 rows, i.e. the reference with capacity 256
        cases = [(0, 0, [("p2p", "p2p", "device", 2.0), ("p2p_ret", "p2p", "device", 2.0),
                         ("p2p_gate", "p2p", "device", 2.0),
                         ("p2p_host", "p2p", "host", 2.0), ("nccl", "nccl", "host", 2.0)]),
                 (300, 300, [("p2p", "p2p", "device", 2.0), ("p2p_host", "p2p", "host", 2.0),
                             ("nccl", "nccl", "host", 2.0)]),
                 (0, 256, [("p2p_bound", "p2p", "device", 0.5)])]
        for cap, ref_cap, variants in cases:
            # single-GPU reference on all tokens
            xa = xs.clone().requires_grad_(True)
            ra = wr.clone().requires_grad_(True)
            a13 = w13.clone().requires_grad_(True)
            a2 = w2.clone().requires_grad_(True)
            ya, _ = moe_ffn(xa, ra, a13, a2, K, ref_cap, True)
            ya.backward(dys)
            for name, transport, layout, bf in variants:
                ep = EPContext(dist.group.WORLD, transport=transport, device=dev, arena_bytes=64 << 20, layout=layout,
                               buffer_factor=bf, epilogue_push=name != "p2p_ret", gate_tiles=name == "p2p_gate")
                for it in range(2):                   # the second pass reuses the device layout's slabs
                    xb = xs[rank * T:(rank + 1) * T].clone().requires_grad_(True)
                    rb = wr.clone().requires_grad_(True)
                    b13 = w13[lo:hi].clone().requires_grad_(True)
                    b2 = w2[lo:hi].clone().requires_grad_(True)
                    ep.begin_step()
                    yb, _ = ep_moe_ffn(xb, rb, b13, b2, K, ep, capacity=cap, renorm=True)
                    yb.backward(dys[rank * T:(rank + 1) * T])
                torch.cuda.synchronize()
                code = C.status()[0]
                C.status_reset()
                # the router gradient of one rank covers its tokens only: sum over ranks
                drb = rb.grad.float().clone()
                dist.all_reduce(drb)
                sl = slice(rank * T, (rank + 1) * T)
                out[(cap, name)] = {
                    "status": code,
                    # pairs beyond the slab bound are dropped (and counted) only in the bounded case
                    "dropped": ((ep.dropped_pairs() > 0) == (name == "p2p_bound"), ep.dropped_pairs()),
                    "y": _close(yb, ya[sl], 2e-2),
                    "dx": _close(xb.grad, xa.grad[sl], 3e-2),
                    "drouter": _close(drb, ra.grad, 3e-2),
                    "dw13": _close(b13.grad, a13.grad[lo:hi], 3e-2),
                    "dw2": _close(b2.grad, a2.grad[lo:hi], 3e-2),
                }
            if cap == 0 and ref_cap == 0:
                # block-scaled fp8 forward expert GEMMs: output within fp8 precision of bf16
                ep = EPContext(dist.group.WORLD, transport="p2p", device=dev, arena_bytes=64 << 20)
                b13, b2 = w13[lo:hi].contiguous(), w2[lo:hi].contiguous()
                ep.set_fp8_weights(b13, b2)
                ep.begin_step()
                with torch.no_grad():
                    yq, _ = ep_moe_ffn(xs[rank * T:(rank + 1) * T], wr, b13, b2, K, ep, capacity=0, renorm=True)
                torch.cuda.synchronize()
                code = C.status()[0]
                C.status_reset()
                out[("fp8", "p2p")] = {"status": code, "y": _close(yq, ya[rank * T:(rank + 1) * T], 8e-2)}
                # training step: fp8 forward and fp8 input gradient through the gate|up experts
                xq_ = xs[rank * T:(rank + 1) * T].clone().requires_grad_(True)
                q13 = w13[lo:hi].clone().requires_grad_(True)
                q2 = w2[lo:hi].clone().requires_grad_(True)
                ep.set_fp8_weights(q13, q2)
                ep.begin_step()
                yq2, _ = ep_moe_ffn(xq_, wr.clone().requires_grad_(True), q13, q2, K, ep, capacity=0, renorm=True)
                yq2.backward(dys[rank * T:(rank + 1) * T])
                torch.cuda.synchronize()
                code = C.status()[0]
                C.status_reset()
                sl = slice(rank * T, (rank + 1) * T)
                out[("fp8_train", "p2p")] = {"status": code, "y": _close(yq2, ya[sl], 8e-2),
                                             "dx": _close(xq_.grad, xa.grad[sl], 1e-1),
                                             "dw13": _close(q13.grad, a13.grad[lo:hi], 1e-1),
                                             "dw2": _close(q2.grad, a2.grad[lo:hi], 1e-1)}
        q.put((rank, out))
    except Exception as e:  # report instead of hanging the parent
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _step_worker(rank, world, port, q, zero_transport="nccl", graph=False):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig, TrainConfig
        from omnicoder.models.lm import build_model
        from omnicoder.ops import _ext
        from omnicoder.parallel.expert_data import ExpertDataParallel
        from omnicoder.training.engine import Trainer, synthetic_batch

        cfg = ModelConfig(name="ep_step", vocab_size=4096, d_model=512, n_layers=2, n_heads=4, ffn_dim=512,
                          tie_embeddings=False, max_seq_len=512,
                          attn=AttentionConfig(kind="mla", kv_lora_rank=256, qk_rope_dim=64, qk_nope_dim=128,
                                               v_head_dim=128),
                          moe=MoEConfig(n_experts=8, top_k=2, ffn_dim=256, n_shared_experts=1, aux_loss_alpha=0.0))
        tc = TrainConfig(lr=1e-3, warmup_steps=0, max_steps=10, grad_clip=1.0)
        ids, lab = synthetic_batch(2 * world, 256, cfg.vocab_size, seed=3, step=0, device=dev)
        ref = build_model(cfg, device=dev, seed=0)
        rt = Trainer(ref, tc)
        n = 5 if graph else 3
        ref_losses = [float(rt.step(ids, lab).loss) for _ in range(n)]
        del rt, ref
        par = ExpertDataParallel(dist.group.WORLD, arena_bytes=64 << 20, zero_transport=zero_transport)
        model = build_model(cfg, device=dev, seed=0, ep=par)
        tr = Trainer(model, tc, par, cuda_graph=graph, graph_warmup=2)
        mine = ids.chunk(world)[rank], lab.chunk(world)[rank]
        losses = []
        for _ in range(n):
            l = tr.step(*mine).loss.detach().float()
            dist.all_reduce(l)
            losses.append(float(l) / world)
        torch.cuda.synchronize()
        C = _ext.load()
        code = C.status()[0]
        C.status_reset()
        q.put((rank, {"ref": ref_losses, "ep": losses, "status": code,
                      "graphed": tr._graph is not None, "graph_error": tr.graph_error}))
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _step_worker_p2p_zero(rank, world, port, q):
    _step_worker(rank, world, port, q, "p2p")


def _step_worker_graph(rank, world, port, q):
    _step_worker(rank, world, port, q, "nccl", graph=True)


def _zero_worker(rank, world, port, q):
    """ZeroAdamW with the peer-memory transport against the NCCL one: same rank-specific
    gradients (produced through autograd, so the bucket hooks fire), three steps each."""
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from omnicoder.ops import _ext
        from omnicoder.parallel.zero import ZeroAdamW
        g0 = torch.Generator().manual_seed(0)
        shapes = [(256, 192), (64,), (1000,), (128, 40), (7, 9)]
        base = [torch.randn(s, generator=g0).to(dev, torch.bfloat16) for s in shapes]
        finals = {}
        for tr in ("nccl", "p2p"):
            params = [torch.nn.Parameter(b.clone()) for b in base]
            opt = ZeroAdamW(params, [], dist.group.WORLD, lr=1e-2, weight_decay=0.1, max_grad_norm=0.5,
                            bucket_bytes=96 * 1024, transport=tr)
            for step in range(3):
                g = torch.Generator().manual_seed(100 + 10 * step + rank)
                coef = [torch.randn(s, generator=g).to(dev) for s in shapes]
                loss = sum((p.float() * c).sum() for p, c in zip(params, coef))
                loss.backward()
                opt.step()
            torch.cuda.synchronize()
            finals[tr] = [p.detach().float().cpu() for p in params]
        C = _ext.load()
        code = C.status()[0]
        C.status_reset()
        err = max(float(((a - b).abs() / (a.abs() + 1.0)).max()) for a, b in zip(finals["nccl"], finals["p2p"]))
        moved = max(float((a - b.float().cpu()).abs().max()) for a, b in zip(finals["p2p"], base))
        q.put((rank, {"err": err, "moved": moved, "status": code}))
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def _run(target, world=2, timeout=600):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(world):
            r, v = q.get(timeout=timeout)
            res[r] = v
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    return res


def _need_gpus(n):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def test_ep_layer_p2p_matches_single_gpu():
    _need_gpus(2)
    res = _run(_layer_worker)
    for rank, out in res.items():
        assert isinstance(out, dict), out
        for key, checks in out.items():
            assert checks["status"] == 0, (rank, key, checks)
            for name, (ok, err) in ((k, v) for k, v in checks.items() if k != "status"):
                assert ok, (rank, key, name, err)


def test_ep_dp_train_step_matches_single_gpu():
    _need_gpus(2)
    res = _run(_step_worker)
    for rank, out in res.items():
        assert isinstance(out, dict), out
        assert out["status"] == 0
        for a, b in zip(out["ref"], out["ep"]):
            assert abs(a - b) < 2e-2 * max(1.0, abs(a)), out


@pytest.mark.parametrize("world", [1, 2])
def test_zero_p2p_optimizer_matches_nccl(world):
    """Fused peer-memory reduce-scatter + AdamW + weight push gives the NCCL ZeRO-1 result."""
    _need_gpus(world)
    res = _run(_zero_worker, world=world)
    for rank, out in res.items():
        assert isinstance(out, dict), out
        assert out["status"] == 0 and out["moved"] > 1e-3, out
        assert out["err"] <= 1e-2, out        # within one bf16 rounding step


def test_ep_dp_train_step_with_p2p_zero_matches_single_gpu():
    _need_gpus(2)
    res = _run(_step_worker_p2p_zero)
    for rank, out in res.items():
        assert isinstance(out, dict), out
        assert out["status"] == 0
        for a, b in zip(out["ref"], out["ep"]):
            assert abs(a - b) < 2e-2 * max(1.0, abs(a)), out


def test_ep_dp_train_step_cuda_graph_matches_single_gpu():
    """Forward + backward of the expert x data parallel step captured as one CUDA graph per
    rank (device-side expert exchange and barriers; ZeRO-1 reductions after the replay): the
    replayed steps give the single-GPU losses."""
    _need_gpus(2)
    res = _run(_step_worker_graph)
    for rank, out in res.items():
        assert isinstance(out, dict), out
        assert out["status"] == 0
        assert out["graphed"], out["graph_error"]
        for a, b in zip(out["ref"], out["ep"]):
            assert abs(a - b) < 2e-2 * max(1.0, abs(a)), out


def _decode_worker(rank, world, port, q):
    """Expert-parallel inference (device layout, shared slabs, graphed decode steps) against a
    full replica of the same weights on this rank's prompts."""
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig
        from omnicoder.inference.graphs import GraphedStep
        from omnicoder.inference.kv_cache import KVCache
        from omnicoder.models.lm import build_model
        from omnicoder.ops import _ext
        from omnicoder.parallel.expert_data import ExpertDataParallel

        cfg = ModelConfig(name="ep_dec", vocab_size=4096, d_model=512, n_layers=2, n_heads=4, ffn_dim=512,
                          tie_embeddings=False, max_seq_len=1024,
                          attn=AttentionConfig(kind="mla", kv_lora_rank=256, qk_rope_dim=64, qk_nope_dim=128,
                                               v_head_dim=128),
                          moe=MoEConfig(n_experts=8, top_k=2, ffn_dim=256, n_shared_experts=1))
        full = build_model(cfg, device=dev, seed=0).eval().prepare_inference()
        par = ExpertDataParallel(dist.group.WORLD, arena_bytes=64 << 20)
        epm = build_model(cfg, device=dev, seed=0, ep=par).eval().prepare_inference()
        B, S = 8, 256
        g = torch.Generator().manual_seed(50 + rank)
        ids = torch.randint(0, cfg.vocab_size, (B, S), generator=g).to(dev)
        ca = KVCache(cfg, B, S + 16, dev, kv_dtype="int8")
        cb = KVCache(cfg, B, S + 16, dev, kv_dtype="int8")
        errs = []
        with torch.no_grad():
            la = full.forward_cached(ids, ca, prefill=True, last_only=True)[:, -1]
            lb = epm.forward_cached(ids, cb, prefill=True, last_only=True)[:, -1]
            errs.append(_close(lb, la, 3e-2))
            step = GraphedStep(epm, cb)
            tok = la.argmax(-1)
            for _ in range(4):
                la = full.forward_cached(tok[:, None], ca)[:, -1]
                lb = step(tok[:, None])[:, -1]
                errs.append(_close(lb, la, 3e-2))
                tok = la.argmax(-1)
        torch.cuda.synchronize()
        C = _ext.load()
        code = C.status()[0]
        C.status_reset()
        q.put((rank, {"errs": errs, "status": code, "dropped": par.ep.dropped_pairs()}))
    except Exception as e:
        q.put((rank, repr(e)))
        raise
    finally:
        dist.destroy_process_group()


def test_ep_inference_prefill_and_graphed_decode_match_replica():
    _need_gpus(2)
    res = _run(_decode_worker)
    for rank, out in res.items():
        assert isinstance(out, dict), out
        assert out["status"] == 0 and out["dropped"] == 0, out
        for ok, err in out["errs"]:
            assert ok, (rank, out["errs"])
