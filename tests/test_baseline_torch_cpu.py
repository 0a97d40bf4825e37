"""The plain PyTorch + torch.distributed comparison build of the MoE pretraining step
(omnicoder.baselines.torch_nccl) on CPU ranks (gloo): expert parallel x data parallel
with ZeRO-1 over 2 ranks must train exactly like one process on the concatenated batch,
and one process must compute the same MoE layer as this package's torch oracle."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig, TrainConfig


def _cfg() -> ModelConfig:
    return ModelConfig(name="baseline_test", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=64,
                       tie_embeddings=False, max_seq_len=64,
                       attn=AttentionConfig(kind="mla", kv_lora_rank=32, qk_rope_dim=8, qk_nope_dim=16,
                                            v_head_dim=16),
                       moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=32, n_shared_experts=1, aux_loss_alpha=0.0))


def _tcfg():
    return TrainConfig(lr=1e-3, warmup_steps=0, max_steps=10, grad_clip=1.0, weight_decay=0.1, eps=1e-6,
                       betas=(0.9, 0.95))


def _load_slice(dst, full, lo, hi):
    """Copy the single-process model's weights into an expert-parallel replica (experts [lo, hi))."""
    src = dict(full.named_parameters())
    with torch.no_grad():
        for n, p in dst.named_parameters():
            w = src[n]
            if n.endswith("moe.w13") or n.endswith("moe.w2"):
                w = w[lo:hi]
            p.copy_(w)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from omnicoder.baselines.torch_nccl import TorchMoELM, TorchTrainer
        cfg = _cfg()
        g = torch.Generator().manual_seed(7)
        ids = torch.randint(0, 300, (2 * world, 32), generator=g)
        lab = torch.randint(0, 300, (2 * world, 32), generator=g)
        ref = TorchMoELM(cfg, "cpu", torch.float32, group=None, seed=0)
        model = TorchMoELM(cfg, "cpu", torch.float32, group=dist.group.WORLD, seed=1)
        El = cfg.moe.n_experts // world
        _load_slice(model, ref, rank * El, (rank + 1) * El)
        rt = TorchTrainer(ref, _tcfg())
        tr = TorchTrainer(model, _tcfg(), dist.group.WORLD)
        ref_l, mine_l = [], []
        for _ in range(3):
            ref_l.append(float(rt.step(ids, lab)))
            loss = tr.step(ids.chunk(world)[rank], lab.chunk(world)[rank])
            dist.all_reduce(loss)
            mine_l.append(float(loss) / world)
        err = 0.0
        src = dict(ref.named_parameters())
        for n, p in model.named_parameters():
            w = src[n]
            if n.endswith("moe.w13") or n.endswith("moe.w2"):
                w = w[rank * El:(rank + 1) * El]
            err = max(err, float((p - w).abs().max()))
        q.put((rank, ref_l, mine_l, err))
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_torch_baseline_ep_dp_matches_single_process():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, ref_l, mine_l, err in res:
        assert all(abs(a - b) < 1e-4 for a, b in zip(ref_l, mine_l)), (rank, ref_l, mine_l)
        assert ref_l[-1] < ref_l[0]
        assert err < 1e-5, (rank, err)


def test_torch_baseline_moe_matches_torch_oracle():
    """One process: the baseline's routed + shared expert layer equals this package's torch
    MoE oracle (same router, top-k renormalised, dropless) on the same weights."""
    from omnicoder.baselines.torch_nccl import MoE
    from omnicoder.ops.gemm import interleave_gate_up
    from omnicoder.ops.moe import moe_ffn_torch
    cfg = _cfg()
    torch.manual_seed(0)
    m = MoE(cfg, "cpu", torch.float32)
    y = torch.randn(50, cfg.d_model)
    out, _ = m(y)
    Fe = cfg.moe.ffn_dim
    w13 = torch.stack([interleave_gate_up(m.w13[e, :Fe], m.w13[e, Fe:]) for e in range(m.El)])
    Fs = m.s2.shape[1]
    s13 = interleave_gate_up(m.s13[:Fs], m.s13[Fs:])
    from omnicoder.ops import swiglu_mlp
    shared = swiglu_mlp(y, s13, m.s2)
    want, _ = moe_ffn_torch(y, m.router, w13, m.w2, cfg.moe.top_k, 0, True, add=shared)
    torch.testing.assert_close(out, want, rtol=1e-4, atol=1e-5)


def _tp_cfg():
    return ModelConfig(name="tp_base", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128,
                       tie_embeddings=False, max_seq_len=64, attn=AttentionConfig(kind="gqa", n_kv_heads=2))


def _tp_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from omnicoder.baselines.torch_tp import TorchDenseTPLM, TorchTPTrainer
        cfg = _tp_cfg()
        tc = TrainConfig(lr=1e-3, warmup_steps=0, max_steps=10, grad_clip=1.0, weight_decay=0.1, eps=1e-6,
                         grad_accum=2)
        ref = TorchDenseTPLM(cfg, "cpu", None, torch.float32, seed=0)
        model = TorchDenseTPLM(cfg, "cpu", dist.group.WORLD, torch.float32, seed=1)
        hd, H, Hk, Fd = cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, cfg.ffn_dim
        h0, h1 = rank * H // world, (rank + 1) * H // world
        k0, k1 = rank * Hk // world, (rank + 1) * Hk // world
        f0, f1 = rank * Fd // world, (rank + 1) * Fd // world
        with torch.no_grad():
            model.embed.copy_(ref.embed)
            model.head.copy_(ref.head)
            model.nf.copy_(ref.nf)
            for a, b in zip(model.blocks, ref.blocks):
                w = b.wqkv
                a.wqkv.copy_(torch.cat([w[h0 * hd:h1 * hd], w[(H + k0) * hd:(H + k1) * hd],
                                        w[(H + Hk + k0) * hd:(H + Hk + k1) * hd]]))
                a.wo.copy_(b.wo[:, h0 * hd:h1 * hd])
                a.w13.copy_(torch.cat([b.w13[f0:f1], b.w13[Fd + f0:Fd + f1]]))
                a.w2.copy_(b.w2[:, f0:f1])
                a.n1.copy_(b.n1)
                a.n2.copy_(b.n2)
        g = torch.Generator().manual_seed(3)
        ids = torch.randint(0, 300, (2, 32), generator=g)
        lab = torch.randint(0, 300, (2, 32), generator=g)
        rt, tr = TorchTPTrainer(ref, tc), TorchTPTrainer(model, tc)
        out = [(float(rt.step(ids, lab)), float(tr.step(ids, lab))) for _ in range(3)]
        err = float((model.blocks[0].wo - ref.blocks[0].wo[:, h0 * hd:h1 * hd]).abs().max())
        q.put((rank, out, err))
    finally:
        dist.destroy_process_group()


def test_torch_tp_baseline_matches_single_process():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_tp_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    for rank, out, err in res:
        for a, b in out:
            assert abs(a - b) < 1e-4, (rank, out)
        assert out[-1][0] < out[0][0]
        assert err < 1e-5, (rank, err)
