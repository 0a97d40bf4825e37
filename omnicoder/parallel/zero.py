"""ZeRO-1 AdamW over a data-parallel group, with bucketed gradient
reduce-scatter overlapped with the backward pass.

Replicated ("dense") parameters are packed into a few flat bf16 buckets, in
reverse registration order so that buckets fill in the order backward produces
gradients.  Each parameter becomes a view into its bucket.  A
post-accumulate-grad hook copies the fresh gradient into the bucket's flat
gradient buffer and releases it; when the last gradient of a bucket arrives the
bucket's reduce-scatter is launched asynchronously (NCCL runs it on its own
stream while backward continues).  Each rank keeps fp32 master weights and
AdamW moments only for its 1/world shard of every bucket; the update kernel
writes the new bf16 shard straight into the bucket, which is then all-gathered
in place.

Expert-parallel parameters (one owner per expert) are not reduced: their
gradients already contain every rank's tokens.  They take a plain local AdamW
step with the same global-norm clip (the squared norm of every shard and every
expert gradient is summed over the group on the device, no host sync).

Weight decay skips 1-D parameters (norm weights); those live in their own
buckets.

transport="p2p" (CUDA, one process per GPU of an NVLink box) keeps every bucket's
gradients and bf16 parameters in peer-mapped symmetric memory and replaces the
NCCL collectives and the separate norm / update kernels: when a bucket's last
gradient arrives, a side stream runs a device barrier over the group and the
fused reduce-scatter (each rank sums its shard straight from every rank's
bucket, scales it and accumulates its squared norm); step() then all-reduces
the one clip-norm scalar and runs the fused AdamW update, which stores the new
bf16 shard into every rank's parameter bucket (the all-gather), followed by a
closing device barrier.  The update rule is torch.optim.AdamW's, the optimiser of the
reference trainer (src/omnicoder/training/pretrain.py:582); the reference has
no sharded optimiser or gradient synchronisation at all.
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist

from ..ops import _ext


class _Bucket:
    def __init__(self, params, world, rank, device, dtype, decay, symm=None):
        self.params = params
        self.decay = decay
        n = sum(p.numel() for p in params)
        quantum = world * 64
        self.n_pad = max(quantum, (n + quantum - 1) // quantum * quantum)
        self.shard = self.n_pad // world
        self.lo = rank * self.shard
        if symm is None:
            self.flat_p = torch.zeros(self.n_pad, device=device, dtype=dtype)
            self.flat_g = torch.zeros(self.n_pad, device=device, dtype=dtype)
        else:
            # peer-mapped: [flat_p | flat_g], every rank's copy addressable from this process
            region = symm.alloc([2 * self.n_pad * 2] * world)
            both = region.view(dtype, 2 * self.n_pad)
            both.zero_()
            self.flat_p, self.flat_g = both[:self.n_pad], both[self.n_pad:]
            self.p_ptrs = list(region.ptrs)
            self.g_ptrs = [ptr + self.n_pad * 2 for ptr in region.ptrs]
            self.shard_gf = torch.zeros(self.shard, device=device, dtype=torch.float32)
        self.offset = {}
        o = 0
        with torch.no_grad():
            for p in params:
                self.flat_p[o:o + p.numel()].copy_(p.data.reshape(-1))
                p.data = self.flat_p[o:o + p.numel()].view_as(p)
                self.offset[p] = o
                o += p.numel()
        self.master = self.flat_p[self.lo:self.lo + self.shard].float().clone()
        self.m = torch.zeros_like(self.master)
        self.v = torch.zeros_like(self.master)
        self.shard_g = torch.zeros(self.shard, device=device, dtype=dtype)
        self.ready = 0
        self.got = set()
        self.work = None


class ZeroAdamW:
    def __init__(self, dense_params, expert_params, group=None, lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                 weight_decay=0.0, max_grad_norm=0.0, bucket_bytes: int = 128 << 20, expert_grad_scale: float = 1.0,
                 transport: str = "nccl"):
        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if transport not in ("nccl", "p2p"):
            raise ValueError(f"unknown ZeRO transport {transport!r}")
        self.p2p = transport == "p2p"
        self.lr, self.betas, self.eps, self.wd = lr, tuple(betas), eps, weight_decay
        self.max_grad_norm = max_grad_norm
        self.expert_grad_scale = expert_grad_scale
        self.step_count = 0
        dense = [p for p in dense_params if p.requires_grad]
        self.device = dense[0].device if dense else (expert_params[0].device if expert_params else torch.device("cpu"))
        self.cuda = self.device.type == "cuda"
        dtype = dense[0].dtype if dense else torch.float32
        if self.p2p and not self.cuda:
            raise ValueError("the peer-memory ZeRO transport needs CUDA tensors")
        self.symm = None
        if self.p2p:
            from .symm import SymmArena
            total = sum(p.numel() for p in dense) * 4 + 8 * 4096
            self.symm = SymmArena(self.group, self.device, chunk_bytes=total)   # bucket storage + barrier flags
            self.side = torch.cuda.Stream(self.device)
        self.buckets: list[_Bucket] = []
        for decay in (True, False):
            group_ps = [p for p in reversed(dense) if (p.dim() > 1) == decay]
            cur, nbytes = [], 0
            for p in group_ps:
                cur.append(p)
                nbytes += p.numel() * p.element_size()
                if nbytes >= bucket_bytes:
                    self.buckets.append(_Bucket(cur, self.world, self.rank, self.device, dtype, decay, self.symm))
                    cur, nbytes = [], 0
            if cur:
                self.buckets.append(_Bucket(cur, self.world, self.rank, self.device, dtype, decay, self.symm))
        self._bucket_of = {p: b for b in self.buckets for p in b.params}
        # every rank starts from rank 0's replica
        for b in self.buckets:
            dist.broadcast(b.flat_p, src=dist.get_global_rank(self.group, 0) if self.group is not dist.group.WORLD
                           else 0, group=self.group)
            b.master.copy_(b.flat_p[b.lo:b.lo + b.shard].float())
        self.experts = [p for p in expert_params if p.requires_grad]
        self.estate = []
        for p in self.experts:
            master = p.detach().float().clone()
            self.estate.append({"master": master, "m": torch.zeros_like(master), "v": torch.zeros_like(master)})
        self._accumulating = False
        self._first_micro = True
        # deferred mode (CUDA-graph replay of forward + backward): the hooks only write the
        # gradients into the buckets (those copies are what a graph captures); step() launches
        # every bucket's reduction
        self.defer = False
        self._norm = torch.zeros(1, device=self.device, dtype=torch.float32)
        for p in dense:
            p.register_post_accumulate_grad_hook(self._hook)

    # ------------------------------------------------------------------
    def set_micro(self, first: bool, last: bool):
        """Gradient accumulation: hooks add into the buckets, reduce only after the last micro-batch."""
        self._first_micro = first
        self._accumulating = not last

    def _hook(self, p: torch.Tensor):
        b = self._bucket_of[p]
        o = b.offset[p]
        dst = b.flat_g[o:o + p.numel()]
        g = p.grad.reshape(-1)
        if self._first_micro:
            dst.copy_(g)
        else:
            dst.add_(g)
        p.grad = None
        if self.defer:
            return
        b.got.add(p)
        b.ready += 1
        if b.ready == len(b.params) and not self._accumulating:
            self._launch(b)

    def _launch(self, b: _Bucket):
        if self.p2p:
            # every rank's bucket gradient is complete -> sum this rank's shard from all of them
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream(self.device))
            with torch.cuda.stream(self.side):
                self.side.wait_event(ev)
                self.symm.barrier()
                _ext.load().zero_rs(b.g_ptrs, b.lo, b.shard, 1.0 / self.world, b.shard_gf,
                                    self._norm if self.max_grad_norm > 0 else None)
            b.work = True
            return
        b.work = dist.reduce_scatter_tensor(b.shard_g, b.flat_g, group=self.group, async_op=True)

    def zero_grad(self, set_to_none: bool = True):
        for p in self.experts:
            p.grad = None

    # ------------------------------------------------------------------
    @torch.no_grad()
    def step(self, lr: float | None = None):
        if lr is not None:
            self.lr = lr
        self.step_count += 1
        if self.defer:                    # every bucket was filled by the replayed backward
            for b in self.buckets:
                if b.work is None:
                    self._launch(b)
        if self.p2p:
            return self._step_p2p()
        for b in self.buckets:
            if b.work is None:            # some parameters of the bucket received no gradient this step
                for p in b.params:
                    if p not in b.got:
                        o = b.offset[p]
                        b.flat_g[o:o + p.numel()].zero_()
                self._launch(b)
        for b in self.buckets:
            b.work.wait()
            b.work = None
            b.ready = 0
            b.got = set()
        gs_dense = 1.0 / self.world
        t = self.step_count
        b1, b2 = self.betas
        if self.cuda:
            C = _ext.load()
            norm = None
            if self.max_grad_norm > 0:
                self._norm.zero_()
                for b in self.buckets:
                    C.sq_norm(b.shard_g, gs_dense, self._norm)
                for p in self.experts:
                    if p.grad is not None:
                        C.sq_norm(p.grad.to(torch.bfloat16).contiguous(), self.expert_grad_scale, self._norm)
                dist.all_reduce(self._norm, group=self.group)
                norm = self._norm
            for b in self.buckets:
                C.adamw(b.master, b.m, b.v, b.shard_g, b.flat_p[b.lo:b.lo + b.shard], self.lr, b1, b2, self.eps,
                        self.wd if b.decay else 0.0, t, gs_dense, norm, self.max_grad_norm)
            for p, st in zip(self.experts, self.estate):
                if p.grad is None:
                    continue
                C.adamw(st["master"], st["m"], st["v"], p.grad.to(torch.bfloat16).contiguous(), p.data, self.lr, b1,
                        b2, self.eps, self.wd if p.dim() > 1 else 0.0, t, self.expert_grad_scale, norm,
                        self.max_grad_norm)
        else:
            clip = 1.0
            if self.max_grad_norm > 0:
                tot = torch.zeros(1)
                for b in self.buckets:
                    tot += (b.shard_g.float() * gs_dense).pow(2).sum()
                for p in self.experts:
                    if p.grad is not None:
                        tot += (p.grad.float() * self.expert_grad_scale).pow(2).sum()
                dist.all_reduce(tot, group=self.group)
                clip = min(1.0, self.max_grad_norm / (math.sqrt(float(tot)) + 1e-6))
            for b in self.buckets:
                _adamw_cpu(b.master, b.m, b.v, b.shard_g.float() * (gs_dense * clip), self.lr, b1, b2, self.eps,
                           self.wd if b.decay else 0.0, t)
                b.flat_p[b.lo:b.lo + b.shard].copy_(b.master)
            for p, st in zip(self.experts, self.estate):
                if p.grad is None:
                    continue
                _adamw_cpu(st["master"], st["m"], st["v"], p.grad.float() * (self.expert_grad_scale * clip), self.lr,
                           b1, b2, self.eps, self.wd if p.dim() > 1 else 0.0, t)
                p.data.copy_(st["master"])
        for b in self.buckets:
            dist.all_gather_into_tensor(b.flat_p, b.flat_p[b.lo:b.lo + b.shard].clone() if not self.cuda
                                        else b.flat_p[b.lo:b.lo + b.shard], group=self.group)

    def _step_p2p(self):
        C = _ext.load()
        cur = torch.cuda.current_stream(self.device)
        for b in self.buckets:
            if b.work is None:            # some parameters of the bucket received no gradient this step
                for p in b.params:
                    if p not in b.got:
                        o = b.offset[p]
                        b.flat_g[o:o + p.numel()].zero_()
                self._launch(b)
        cur.wait_stream(self.side)
        for b in self.buckets:
            b.work = None
            b.ready = 0
            b.got = set()
        t = self.step_count
        b1, b2 = self.betas
        norm = None
        if self.max_grad_norm > 0:
            for p in self.experts:
                if p.grad is not None:
                    C.sq_norm(p.grad.to(torch.bfloat16).contiguous(), self.expert_grad_scale, self._norm)
            dist.all_reduce(self._norm, group=self.group)
            norm = self._norm
        for b in self.buckets:
            C.zero_adamw_push(b.master, b.m, b.v, b.shard_gf, b.p_ptrs, b.lo, self.lr, b1, b2, self.eps,
                              self.wd if b.decay else 0.0, t, norm, self.max_grad_norm)
        for p, st in zip(self.experts, self.estate):
            if p.grad is None:
                continue
            C.adamw(st["master"], st["m"], st["v"], p.grad.to(torch.bfloat16).contiguous(), p.data, self.lr, b1,
                    b2, self.eps, self.wd if p.dim() > 1 else 0.0, t, self.expert_grad_scale, norm,
                    self.max_grad_norm)
        self.symm.barrier()               # every rank's parameter bucket is complete before the next forward
        if self.max_grad_norm > 0:
            self._norm.zero_()            # the next step's reduce-scatters accumulate into it

    # ------------------------------------------------------------------
    def state_dict(self) -> dict:
        """This rank's shard of the optimiser state (save one file per rank)."""
        return {"step": self.step_count, "rank": self.rank, "world": self.world,
                "buckets": [{"master": b.master.cpu(), "m": b.m.cpu(), "v": b.v.cpu()} for b in self.buckets],
                "experts": [{k: v.cpu() for k, v in s.items()} for s in self.estate]}

    def load_state_dict(self, sd: dict):
        if sd["world"] != self.world:
            raise ValueError("sharded optimiser state was saved with a different world size")
        self.step_count = int(sd["step"])
        for b, s in zip(self.buckets, sd["buckets"]):
            b.master.copy_(s["master"])
            b.m.copy_(s["m"])
            b.v.copy_(s["v"])
            b.flat_p[b.lo:b.lo + b.shard].copy_(b.master.to(b.flat_p.dtype))
        for st, s in zip(self.estate, sd["experts"]):
            for k in st:
                st[k].copy_(s[k])
        for p, st in zip(self.experts, self.estate):
            p.data.copy_(st["master"].to(p.dtype))
        for b in self.buckets:
            dist.all_gather_into_tensor(b.flat_p, b.flat_p[b.lo:b.lo + b.shard].clone(), group=self.group)


def _adamw_cpu(w, m, v, g, lr, b1, b2, eps, wd, t):
    m.mul_(b1).add_(g, alpha=1 - b1)
    v.mul_(b2).addcmul_(g, g, value=1 - b2)
    w.mul_(1 - lr * wd)
    denom = (v.sqrt() / math.sqrt(1 - b2 ** t)).add_(eps)
    w.addcdiv_(m, denom, value=-lr / (1 - b1 ** t))
