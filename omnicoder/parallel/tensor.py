"""Tensor parallelism with sequence parallelism (dense spec models).

Layout inside a TP group of N ranks:
  * between blocks the residual stream is sharded along tokens: rank r holds
    tokens [r T/N, (r+1) T/N) of the micro-batch (T = batch * seq);
  * attention: all-gather of the normalised tokens -> each rank projects its
    n_heads / N query heads and n_kv_heads / N kv heads, attends over full
    sequences, projects back with its slice of the output projection -> partial
    sums reduce-scattered along tokens (+ residual);
  * SwiGLU MLP: all-gather -> gate/up for F / N hidden features -> down ->
    reduce-scatter;
  * embeddings, norms and the LM head stay replicated; each rank applies them to
    its own tokens, so their gradients are summed over the group.

Collectives: `all_gather_seq` / `reduce_scatter_seq` are autograd functions
(their backward is the other collective).  The NCCL path uses
all_gather_into_tensor / reduce_scatter_tensor; on CPU the same code runs on
gloo (the multi-process tests).

The reference has no tensor parallelism (only a vLLM adapter argument for an
external model, src/omnicoder/inference/runtimes/vllm_adapter.py:13-33).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


class TPContext:
    def __init__(self, group=None):
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)

    def shard(self, n: int, what: str) -> tuple[int, int]:
        if n % self.world:
            raise ValueError(f"{what} ({n}) must divide by the tensor-parallel size {self.world}")
        per = n // self.world
        return self.rank * per, (self.rank + 1) * per


def _ag(x: torch.Tensor, group, world: int) -> torch.Tensor:
    out = x.new_empty((x.shape[0] * world,) + tuple(x.shape[1:]))
    dist.all_gather_into_tensor(out, x.contiguous(), group=group)
    return out


def _rs(x: torch.Tensor, group, world: int) -> torch.Tensor:
    out = x.new_empty((x.shape[0] // world,) + tuple(x.shape[1:]))
    dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
    return out


class _AllGatherSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return _ag(x, tp.group, tp.world)

    @staticmethod
    def backward(ctx, g):
        return _rs(g, ctx.tp.group, ctx.tp.world), None


class _ReduceScatterSeq(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, tp):
        ctx.tp = tp
        return _rs(x, tp.group, tp.world)

    @staticmethod
    def backward(ctx, g):
        return _ag(g, ctx.tp.group, ctx.tp.world), None


def all_gather_seq(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    return x if tp.world == 1 else _AllGatherSeq.apply(x, tp)


def reduce_scatter_seq(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    return x if tp.world == 1 else _ReduceScatterSeq.apply(x, tp)


def scatter_seq(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """This rank's token shard of a replicated [T, ...] tensor (no communication)."""
    lo, hi = tp.shard(x.shape[0], "token count")
    return x[lo:hi]


class TensorParallel:
    """Trainer-facing layout object: optimizer over local parameters, gradient
    all-reduce of the replicated ones over the TP group (bucketed, one NCCL call
    per bucket)."""

    def __init__(self, group=None, bucket_bytes: int = 64 << 20):
        self.tp = TPContext(group)
        self.group, self.rank, self.world = self.tp.group, self.tp.rank, self.tp.world
        self.bucket_bytes = bucket_bytes

    def make_optimizer(self, model, tcfg):
        from ..ops import FusedAdamW
        self.replicated = [p for n, p in model.named_parameters() if not getattr(p, "tp_sharded", False)]
        self.sharded = [p for n, p in model.named_parameters() if getattr(p, "tp_sharded", False)]
        self.max_grad_norm = tcfg.grad_clip
        # clipping is applied here (global norm over the group), not inside the optimiser
        return FusedAdamW(model.parameters(), lr=tcfg.lr, betas=tuple(tcfg.betas), eps=tcfg.eps,
                          weight_decay=tcfg.weight_decay, max_grad_norm=0.0)

    def before_forward(self, micro: int, n_micro: int):
        pass

    @torch.no_grad()
    def sync_grads(self):
        ps = [p for p in self.replicated if p.grad is not None]
        i = 0
        while i < len(ps):
            j, nb = i, 0
            while j < len(ps) and (nb == 0 or nb + ps[j].numel() * ps[j].grad.element_size() <= self.bucket_bytes):
                nb += ps[j].numel() * ps[j].grad.element_size()
                j += 1
            flat = torch.cat([p.grad.reshape(-1) for p in ps[i:j]])
            dist.all_reduce(flat, group=self.group)
            o = 0
            for p in ps[i:j]:
                p.grad.copy_(flat[o:o + p.numel()].view_as(p.grad))
                o += p.numel()
            i = j

    def sync_and_step(self, model, opt, lr: float):
        """Every rank back-propagated the mean loss of its own tokens: sum the replicated
        gradients over the group, then scale every gradient by 1/N (the group mean
        loss) and by the global-norm clip factor."""
        self.sync_grads()
        scale = 1.0 / self.world
        if self.max_grad_norm > 0:
            dev = next((p.grad.device for p in self.sharded + self.replicated if p.grad is not None), None)
            sh = torch.zeros((), device=dev)
            for p in self.sharded:
                if p.grad is not None:
                    sh += p.grad.float().pow(2).sum()
            dist.all_reduce(sh, group=self.group)
            for p in self.replicated:
                if p.grad is not None:
                    sh += p.grad.float().pow(2).sum()
            norm = float(sh.sqrt()) * scale
            scale *= min(1.0, self.max_grad_norm / (norm + 1e-6))
        opt.step(lr=lr, grad_scale=scale)
