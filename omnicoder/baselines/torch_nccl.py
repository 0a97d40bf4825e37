"""Plain PyTorch + NCCL + cuBLAS build of the MoE LM pretraining step.

This is the comparison arm of the training benchmark: the same model, data,
routing and optimiser as :class:`omnicoder.models.lm.OmniLM` under
:class:`omnicoder.training.engine.Trainer`, written only with stock PyTorch
operators, as a competent PyTorch user would write it without custom kernels:

* linears are bf16 ``F.linear`` (cuBLAS), norms ``F.rms_norm``, attention
  ``F.scaled_dot_product_attention`` (causal; PyTorch picks its backend);
* MLA attention in its training form: q [T, H, nope+rope], latent KV
  projection + RMSNorm, up-projection to per-head keys / values, a shared rope
  key broadcast over heads;
* routed experts: softmax router, top-k with renormalisation, pairs sorted by
  expert, ``torch._grouped_mm`` (one grouped bf16 GEMM per projection) with the
  SwiGLU between them, a batched weighted sum back to tokens; a shared expert;
* expert parallelism over the process group: routing counts exchanged with
  ``all_to_all_single``, tokens dispatched and returned with
  ``all_to_all_single`` (autograd runs the transposed exchange in backward);
* ZeRO-1 AdamW: dense (replicated) parameters live in flat bf16 buckets whose
  gradient ``reduce_scatter_tensor`` is launched from post-accumulate-grad
  hooks while backward continues; fp32 master weights and moments only for this
  rank's shard, ``torch.optim.AdamW(fused=True)``, global-norm clip,
  ``all_gather_into_tensor`` of the updated bf16 shards; expert parameters
  (one owner each) step locally.

Nothing here imports this package's CUDA extension.  The reference project has
no distributed path of its own (src/omnicoder/tools/torchrun_ep.py:7-18 sets up
a process group and never reduces anything), so this arm stands in for "the
reference's torch.distributed NCCL + cuBLAS build".
"""
from __future__ import annotations

import math

import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..config import ModelConfig, TrainConfig


# ----------------------------------------------------------------------------
# model
# ----------------------------------------------------------------------------
def _param(shape, std, device, dtype):
    t = torch.empty(shape, device=device, dtype=dtype)
    with torch.no_grad():
        t.normal_(0.0, std)
    return nn.Parameter(t)


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Half-split rotation of x [..., T, (H,) rot] by cos / sin [T, 1, rot/2] (or [T, rot/2])."""
    h = x.shape[-1] // 2
    x0, x1 = x[..., :h], x[..., h:]
    return torch.cat([x0 * cos - x1 * sin, x1 * cos + x0 * sin], dim=-1)


class _A2A(torch.autograd.Function):
    """all_to_all_single with its transpose as the backward."""

    @staticmethod
    def forward(ctx, x, send: list, recv: list, group):
        ctx.send, ctx.recv, ctx.group = send, recv, group
        out = x.new_empty((sum(recv),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv, send, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = g.new_empty((sum(ctx.send),) + tuple(g.shape[1:]))
        dist.all_to_all_single(out, g.contiguous(), ctx.send, ctx.recv, group=ctx.group)
        return out, None, None, None


class MLA(nn.Module):
    def __init__(self, cfg: ModelConfig, device, dtype):
        super().__init__()
        a, D, H = cfg.attn, cfg.d_model, cfg.n_heads
        self.H, self.dn, self.dr, self.dv, self.r, self.eps = H, a.qk_nope_dim, a.qk_rope_dim, a.v_head_dim, \
            a.kv_lora_rank, cfg.norm_eps
        s = cfg.init_std
        self.wq = _param((H * (self.dn + self.dr), D), s, device, dtype)
        self.wkv_a = _param((self.r + self.dr, D), s, device, dtype)
        self.kv_norm = nn.Parameter(torch.ones(self.r, device=device, dtype=dtype))
        self.wkv_b = _param((H * (self.dn + self.dv), self.r), s, device, dtype)
        self.wo = _param((D, H * self.dv), s, device, dtype)

    def forward(self, y, B, S, cos, sin):
        T, H, dn, dr = y.shape[0], self.H, self.dn, self.dr
        q = F.linear(y, self.wq).view(T, H, dn + dr)
        q = torch.cat([q[..., :dn], _rope(q[..., dn:], cos[:, None], sin[:, None])], dim=-1)
        kva = F.linear(y, self.wkv_a)
        c = F.rms_norm(kva[:, :self.r], (self.r,), self.kv_norm, self.eps)
        kr = _rope(kva[:, self.r:], cos, sin)                                  # [T, dr], shared by heads
        kv = F.linear(c, self.wkv_b).view(T, H, dn + self.dv)
        k = torch.cat([kv[..., :dn], kr[:, None].expand(T, H, dr)], dim=-1)
        v = kv[..., dn:]
        qb = q.view(B, S, H, -1).transpose(1, 2)
        kb = k.view(B, S, H, -1).transpose(1, 2)
        vb = v.reshape(B, S, H, -1).transpose(1, 2)
        o = F.scaled_dot_product_attention(qb, kb, vb, is_causal=True, scale=1.0 / math.sqrt(dn + dr))
        return F.linear(o.transpose(1, 2).reshape(T, H * self.dv), self.wo)


def _swiglu(y, w13, w2):
    h = F.linear(y, w13)
    f = h.shape[-1] // 2
    return F.linear(F.silu(h[:, :f]) * h[:, f:], w2)


class MoE(nn.Module):
    """Routed SwiGLU experts (this rank's slice when `group` has more than one rank) + shared expert."""

    def __init__(self, cfg: ModelConfig, device, dtype, group=None):
        super().__init__()
        m, D, s = cfg.moe, cfg.d_model, cfg.init_std
        self.E, self.k, self.Fe, self.renorm, self.alpha = m.n_experts, m.top_k, m.ffn_dim, m.renorm_topk, \
            m.aux_loss_alpha
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        if self.E % self.world:
            raise ValueError(f"{self.E} experts do not divide over {self.world} ranks")
        self.El = self.E // self.world
        self.router = _param((self.E, D), s, device, dtype)
        # gate rows [0, F) and up rows [F, 2F) of every local expert
        self.w13 = _param((self.El, 2 * self.Fe, D), s, device, dtype)
        self.w2 = _param((self.El, D, self.Fe), s, device, dtype)
        Fs = m.ffn_dim * m.n_shared_experts
        self.shared = None
        if Fs:
            self.s13 = _param((2 * Fs, D), s, device, dtype)
            self.s2 = _param((D, Fs), s, device, dtype)
            self.shared = True

    def experts(self, x, offs):
        h = torch._grouped_mm(x, self.w13.transpose(-2, -1), offs=offs)
        a = F.silu(h[:, :self.Fe]) * h[:, self.Fe:]
        return torch._grouped_mm(a, self.w2.transpose(-2, -1), offs=offs)

    def forward(self, y):
        T, D = y.shape
        E, k, N, El = self.E, self.k, self.world, self.El
        logits = F.linear(y.float(), self.router.float())
        probs = torch.softmax(logits, dim=-1)
        w, idx = torch.topk(probs, k, dim=-1)
        if self.renorm:
            w = w / w.sum(-1, keepdim=True)
        flat = idx.reshape(-1)
        order = torch.argsort(flat, stable=True)                               # pairs by expert
        counts = torch.bincount(flat, minlength=E)
        xs = y.index_select(0, order // k)
        if N == 1:
            ye = self.experts(xs, counts.cumsum(0).to(torch.int32))
        else:
            # counts exchange, then tokens: the receive side gets source-major blocks of
            # (source, local expert); they are regrouped expert-major for the grouped GEMM
            rc = torch.empty_like(counts)
            dist.all_to_all_single(rc, counts, group=self.group)
            send = counts.view(N, El).sum(1).tolist()
            rcm = rc.view(N, El)
            recv = rcm.sum(1).tolist()
            xr = _A2A.apply(xs, send, recv, self.group)
            nblk = rcm.reshape(-1)
            src_start = nblk.cumsum(0) - nblk                                  # (s, e) order
            dmat = rcm.t().reshape(-1)
            dst_start_t = (dmat.cumsum(0) - dmat).view(El, N).t().reshape(-1)  # (e, s) order, indexed by (s, e)
            tot = int(sum(recv))
            blk = torch.repeat_interleave(torch.arange(N * El, device=y.device), nblk, output_size=tot)
            dst = dst_start_t[blk] + torch.arange(tot, device=y.device) - src_start[blk]
            inv = torch.empty_like(dst)
            inv[dst] = torch.arange(tot, device=y.device)
            ye = self.experts(xr.index_select(0, inv), rcm.sum(0).cumsum(0).to(torch.int32))
            ye = _A2A.apply(ye.index_select(0, dst), recv, send, self.group)
        inv_order = torch.empty_like(order)
        inv_order[order] = torch.arange(order.numel(), device=y.device)
        yp = ye.index_select(0, inv_order).view(T, k, D)
        out = torch.bmm(w.to(y.dtype).unsqueeze(1), yp).squeeze(1)
        if self.shared:
            out = out + _swiglu(y, self.s13, self.s2)
        aux = self.alpha * E * ((counts.float() / (T * k)) * probs.mean(0)).sum()
        return out, aux


class Block(nn.Module):
    def __init__(self, cfg, device, dtype, group):
        super().__init__()
        self.eps, D = cfg.norm_eps, cfg.d_model
        self.n1 = nn.Parameter(torch.ones(D, device=device, dtype=dtype))
        self.attn = MLA(cfg, device, dtype)
        self.n2 = nn.Parameter(torch.ones(D, device=device, dtype=dtype))
        self.moe = MoE(cfg, device, dtype, group)

    def forward(self, h, B, S, cos, sin):
        D = h.shape[-1]
        h = h + self.attn(F.rms_norm(h, (D,), self.n1, self.eps), B, S, cos, sin)
        out, aux = self.moe(F.rms_norm(h, (D,), self.n2, self.eps))
        return h + out, aux


class TorchMoELM(nn.Module):
    """The MoE MLA LM (spec family architecture) in plain PyTorch; `group` shards the experts."""

    def __init__(self, cfg: ModelConfig, device, dtype=torch.bfloat16, group=None, seed: int = 1234):
        super().__init__()
        if cfg.attn.kind != "mla" or not cfg.moe.enabled:
            raise ValueError("the torch baseline models the MLA + routed-expert family")
        torch.manual_seed(seed)
        torch.cuda.manual_seed(seed) if str(device).startswith("cuda") else None
        self.cfg = cfg
        D, V = cfg.d_model, cfg.vocab_size
        self.embed = _param((V, D), cfg.init_std, device, dtype)
        self.blocks = nn.ModuleList([Block(cfg, device, dtype, group) for _ in range(cfg.n_layers)])
        self.nf = nn.Parameter(torch.ones(D, device=device, dtype=dtype))
        self.head = _param((V, D), cfg.init_std, device, dtype)
        a = cfg.attn
        inv = a.rope_theta ** (-torch.arange(0, a.qk_rope_dim, 2, dtype=torch.float64) / a.qk_rope_dim)
        ang = torch.outer(torch.arange(cfg.max_seq_len, dtype=torch.float64) / a.rope_scale, inv)
        self.register_buffer("cos", ang.cos().to(dtype).to(device), persistent=False)
        self.register_buffer("sin", ang.sin().to(dtype).to(device), persistent=False)

    def expert_params(self):
        return [p for b in self.blocks for p in (b.moe.w13, b.moe.w2)]

    def forward(self, ids, labels):
        B, S = ids.shape
        pos = torch.arange(S, device=ids.device).repeat(B)
        cos, sin = self.cos[pos], self.sin[pos]
        h = F.embedding(ids.reshape(-1), self.embed)
        aux = None
        for blk in self.blocks:
            h, a = blk(h, B, S, cos, sin)
            aux = a if aux is None else aux + a
        y = F.rms_norm(h, (h.shape[-1],), self.nf, self.cfg.norm_eps)
        logits = F.linear(y, self.head)
        ce = F.cross_entropy(logits.float(), labels.reshape(-1))
        return ce + aux, ce, aux


# ----------------------------------------------------------------------------
# ZeRO-1 AdamW with torch collectives
# ----------------------------------------------------------------------------
class _FlatBucket:
    """Replicated parameters packed into one flat bf16 buffer (each parameter becomes a view)."""

    def __init__(self, params, world, rank, decay):
        self.params, self.decay = params, decay
        dev, dt = params[0].device, params[0].dtype
        n = sum(p.numel() for p in params)
        q = world * 64
        self.n = (n + q - 1) // q * q
        self.shard = self.n // world
        self.lo = rank * self.shard
        self.flat_p = torch.zeros(self.n, device=dev, dtype=dt)
        self.flat_g = torch.zeros(self.n, device=dev, dtype=dt)
        self.shard_g = torch.zeros(self.shard, device=dev, dtype=dt)
        self.offset, o = {}, 0
        with torch.no_grad():
            for p in params:
                self.flat_p[o:o + p.numel()].copy_(p.data.reshape(-1))
                p.data = self.flat_p[o:o + p.numel()].view_as(p)
                self.offset[p] = o
                o += p.numel()
        self.master = nn.Parameter(self.flat_p[self.lo:self.lo + self.shard].float().clone())
        self.pending = 0
        self.got = set()
        self.work = None


class TorchZeroAdamW:
    """ZeRO-1 AdamW: bucketed bf16 gradient reduce-scatter from backward hooks, fused AdamW
    (torch.optim.AdamW(fused=True)) on fp32 master shards, global-norm clip, all-gather of the
    updated bf16 shards.  Expert parameters (`experts`, one owner each) are stepped locally;
    their gradients are scaled by `expert_grad_scale` (1 / world: the loss is a per-rank mean)."""

    def __init__(self, dense, experts, group, lr, betas, eps, weight_decay, max_grad_norm,
                 bucket_bytes: int = 128 << 20, expert_grad_scale: float = 1.0, chunk_elems: int = 1 << 28):
        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        self.max_grad_norm, self.expert_grad_scale = max_grad_norm, expert_grad_scale
        self.buckets: list[_FlatBucket] = []
        for decay in (True, False):
            cur, nb = [], 0
            for p in reversed([p for p in dense if (p.dim() > 1) == decay]):
                cur.append(p)
                nb += p.numel() * p.element_size()
                if nb >= bucket_bytes:
                    self.buckets.append(_FlatBucket(cur, self.world, self.rank, decay))
                    cur, nb = [], 0
            if cur:
                self.buckets.append(_FlatBucket(cur, self.world, self.rank, decay))
        self.of = {p: b for b in self.buckets for p in b.params}
        if self.world > 1:
            for b in self.buckets:
                dist.broadcast(b.flat_p, src=dist.get_global_rank(group, 0), group=group)
                with torch.no_grad():
                    b.master.copy_(b.flat_p[b.lo:b.lo + b.shard].float())
        for p in dense:
            p.register_post_accumulate_grad_hook(self._hook)
        self.experts = list(experts)
        self.emaster = [nn.Parameter(p.detach().float().clone()) for p in self.experts]
        # fused AdamW over the fp32 masters, in chunks so that the fp32 copies of the
        # gradients exist for one chunk at a time
        masters = [(b.master, b.decay) for b in self.buckets] + [(m, m.dim() > 1) for m in self.emaster]
        self.chunks, cur, n = [], [], 0
        for m, decay in masters:
            cur.append((m, decay))
            n += m.numel()
            if n >= chunk_elems:
                self.chunks.append(cur)
                cur, n = [], 0
        if cur:
            self.chunks.append(cur)
        self.opts = []
        for ch in self.chunks:
            groups = [{"params": [m for m, d in ch if d], "weight_decay": weight_decay},
                      {"params": [m for m, d in ch if not d], "weight_decay": 0.0}]
            self.opts.append(torch.optim.AdamW([g for g in groups if g["params"]], lr=lr, betas=betas, eps=eps,
                                               fused=True))

    def _hook(self, p):
        b = self.of[p]
        o = b.offset[p]
        b.flat_g[o:o + p.numel()].copy_(p.grad.reshape(-1))
        p.grad = None
        b.got.add(p)
        b.pending += 1
        if b.pending == len(b.params):
            self._reduce(b)

    def _reduce(self, b):
        if self.world > 1:
            b.work = dist.reduce_scatter_tensor(b.shard_g, b.flat_g, op=dist.ReduceOp.AVG, group=self.group,
                                                async_op=True)
        else:
            b.shard_g.copy_(b.flat_g)

    @torch.no_grad()
    def step(self, lr: float):
        for b in self.buckets:
            if b.pending != len(b.params):          # parameters without a gradient this step: zeros
                for p in b.params:
                    if p not in b.got:
                        b.flat_g[b.offset[p]:b.offset[p] + p.numel()].zero_()
                self._reduce(b)
            if b.work is not None:
                b.work.wait()
                b.work = None
            b.pending = 0
            b.got = set()
        # global gradient norm over every shard and every expert gradient (device scalars)
        sq = [b.shard_g.float().pow(2).sum() for b in self.buckets]
        sq += [(p.grad.float() * self.expert_grad_scale).pow(2).sum() for p in self.experts if p.grad is not None]
        tot = torch.stack(sq).sum().reshape(1)
        if self.world > 1:
            dist.all_reduce(tot, group=self.group)
        coef = (self.max_grad_norm / (tot.sqrt() + 1e-6)).clamp(max=1.0) if self.max_grad_norm > 0 else None
        grad_src = {id(b.master): (b.shard_g, 1.0) for b in self.buckets}
        for p, m in zip(self.experts, self.emaster):
            grad_src[id(m)] = (p.grad, self.expert_grad_scale)
        for opt, ch in zip(self.opts, self.chunks):
            for m, _ in ch:
                g, s = grad_src[id(m)]
                if g is None:
                    m.grad = None
                    continue
                gf = g.reshape(m.shape).float()
                if s != 1.0:
                    gf.mul_(s)
                if coef is not None:
                    gf.mul_(coef)
                m.grad = gf
            for grp in opt.param_groups:
                grp["lr"] = lr
            opt.step()
            for m, _ in ch:
                m.grad = None
        for b in self.buckets:
            b.flat_p[b.lo:b.lo + b.shard].copy_(b.master)
            if self.world > 1:
                dist.all_gather_into_tensor(b.flat_p, b.flat_p[b.lo:b.lo + b.shard].clone(), group=self.group)
        for p, m in zip(self.experts, self.emaster):
            p.copy_(m)
            p.grad = None


class TorchTrainer:
    """Forward, backward and optimiser step of the plain PyTorch build (same learning-rate
    schedule as omnicoder.training.engine.Trainer)."""

    def __init__(self, model: TorchMoELM, tcfg: TrainConfig, group=None):
        self.model, self.tcfg, self.step_idx = model, tcfg, 0
        experts = model.expert_params()
        eid = {id(p) for p in experts}
        dense = [p for p in model.parameters() if id(p) not in eid]
        world = dist.get_world_size(group) if group is not None else 1
        self.opt = TorchZeroAdamW(dense, experts, group, tcfg.lr, tuple(tcfg.betas), tcfg.eps, tcfg.weight_decay,
                                  tcfg.grad_clip, expert_grad_scale=1.0 / world)

    def step(self, ids, labels):
        from ..ops.optim import cosine_lr
        loss, ce, aux = self.model(ids, labels)
        loss.backward()
        lr = cosine_lr(self.step_idx, self.tcfg.lr, self.tcfg.warmup_steps, self.tcfg.max_steps)
        self.opt.step(lr)
        self.step_idx += 1
        return loss.detach()
