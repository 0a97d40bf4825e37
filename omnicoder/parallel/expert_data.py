"""Expert parallel x data parallel training layout over one process group.

Every rank holds a full replica of the dense parameters (attention, norms,
embeddings, router, shared experts) and 1/world of the routed experts.  The
data-parallel side is ZeRO-1 (:class:`omnicoder.parallel.zero.ZeroAdamW`):
bucketed gradient reduce-scatter overlapped with backward, sharded fp32
master/moments, in-place all-gather of the updated bf16 parameters.  The
expert-parallel side (:mod:`omnicoder.parallel.expert`) moves tokens to the
owner of their expert and back.

    group = dist.group.WORLD
    par = ExpertDataParallel(group)
    model = build_model(cfg, device, seed=0, ep=par)
    trainer = Trainer(model, tcfg, par)

The reference's only multi-GPU entry point (src/omnicoder/tools/torchrun_ep.py)
initialises a process group and never synchronises anything.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .expert import EPContext
from .zero import ZeroAdamW


class ExpertDataParallel:
    def __init__(self, group=None, transport: str = "auto", bucket_bytes: int = 128 << 20,
                 arena_bytes: int = 1 << 30, zero_transport: str = "nccl", layout: str = "device",
                 buffer_factor: float = 2.0):
        """zero_transport: "nccl" (reduce-scatter / all-gather collectives) or "p2p" (the
        reduce-scatter and the updated-weight all-gather fused into the optimiser kernels over
        peer memory, see omnicoder.parallel.zero)."""
        self.group = group if group is not None else dist.group.WORLD
        self.zero_transport = zero_transport
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.ep = EPContext(self.group, transport=transport, arena_bytes=arena_bytes, layout=layout,
                            buffer_factor=buffer_factor)
        self.bucket_bytes = bucket_bytes
        self.opt = None

    @staticmethod
    def arena_bytes_for(cfg, tokens_per_rank: int, world: int, buffer_factor: float = 2.0) -> int:
        """Peer-mapped bytes per rank that the device-layout exchange of one step of `cfg` needs
        (every MoE layer's receive rows / metadata and (token, k) output slots, the shared
        backward slabs, the count board)."""
        import math
        m = cfg.moe
        E, k, D = m.n_experts, m.top_k, cfg.d_model
        El = E // world
        if m.capacity_factor > 0:
            cap = m.capacity(tokens_per_rank * world)
            seg = (cap + 127) // 128 * 128
        else:
            seg = max(128, (math.ceil(buffer_factor * world * tokens_per_rank * k / E) + 127) // 128 * 128)
        R = El * seg
        n_moe = sum(1 for i in range(cfg.n_layers) if cfg.is_moe_layer(i))
        pairs = tokens_per_rank * k
        per_layer = R * D * 2 + R * 16 + pairs * D * 2
        shared = R * D * 2 + pairs * D * 2 + world * E * 4
        return n_moe * (per_layer + 1024) + shared + (1 << 20)

    # ---- model construction -------------------------------------------------
    def expert_slice(self, n_experts: int) -> tuple[int, int]:
        return self.ep.experts_of(n_experts)

    @staticmethod
    def expert_params(model) -> list:
        from ..models.lm import MoEFFN
        out = []
        for m in model.modules():
            if isinstance(m, MoEFFN):
                out += [m.w13, m.w2]
        return out

    # ---- training -----------------------------------------------------------
    def make_optimizer(self, model, tcfg):
        experts = self.expert_params(model)
        eid = {id(p) for p in experts}
        dense = [p for p in model.parameters() if id(p) not in eid]
        self.opt = ZeroAdamW(dense, experts, self.group, lr=tcfg.lr, betas=tuple(tcfg.betas), eps=tcfg.eps,
                             weight_decay=tcfg.weight_decay, max_grad_norm=tcfg.grad_clip,
                             bucket_bytes=self.bucket_bytes, expert_grad_scale=1.0 / self.world,
                             transport=self.zero_transport)
        return self.opt

    def before_forward(self, micro: int, n_micro: int):
        self.ep.begin_step()
        if self.opt is not None:
            self.opt.set_micro(first=micro == 0, last=micro == n_micro - 1)

    def sync_and_step(self, model, opt, lr: float):
        opt.step(lr=lr)

    def graph_capturable(self) -> bool:
        """Forward + backward can be captured as one CUDA graph: the expert exchange runs on the
        device layout (no host synchronisation, fixed slabs, device-epoch barriers)."""
        return self.ep.transport == "p2p" and self.ep.layout == "device" and self.ep.device.type == "cuda"

    def set_deferred_reduce(self, on: bool):
        if self.opt is not None:
            self.opt.defer = on

    def all_reduce_mean(self, t: torch.Tensor) -> torch.Tensor:
        t = t.clone()
        dist.all_reduce(t, group=self.group)
        return t / self.world
