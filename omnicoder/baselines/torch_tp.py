"""Plain PyTorch + NCCL + cuBLAS tensor-parallel (sequence-parallel) build of the dense
GQA LM training step -- the comparison arm of the dense 20B benchmark.

Layout (Megatron-style sequence parallelism over a group of N ranks):
  * between blocks every rank holds T / N tokens of the residual stream;
  * attention: the normalised shard is all-gathered (``all_gather_into_tensor``),
    each rank projects H / N query heads and Hk / N kv heads (bf16 ``F.linear``),
    rotates them (half-split RoPE), runs ``F.scaled_dot_product_attention``
    (causal, GQA) and projects back with its slice of the output projection; the
    partial sums are reduce-scattered (``reduce_scatter_tensor``) to token shards;
  * SwiGLU MLP: all-gather -> F / N hidden features -> reduce-scatter;
  * embeddings, norms and the LM head are replicated and applied to the rank's own
    tokens; their gradients are all-reduced over the group.
Optimiser: ``torch.optim.AdamW(fused=True)`` on fp32 master copies, global-norm clip.
``fp8=True``: the four projections of every block run their forward and input-gradient
GEMMs through ``torch._scaled_mm`` on e4m3 operands with row-wise scales (one fp32 scale
per token row of the activation / gradient and per row of the weight: the plain-PyTorch
fp8 recipe on cuBLAS); weight gradients stay bf16.

Nothing here imports this package's CUDA extension.  The reference has no tensor
parallelism (its only mention is an external vLLM argument,
src/omnicoder/inference/runtimes/vllm_adapter.py:13-33).
"""
from __future__ import annotations


import torch
import torch.distributed as dist
import torch.nn as nn
import torch.nn.functional as F

from ..config import ModelConfig, TrainConfig


class _AG(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, n):
        ctx.group, ctx.n = group, n
        out = x.new_empty((x.shape[0] * n,) + tuple(x.shape[1:]))
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = g.new_empty((g.shape[0] // ctx.n,) + tuple(g.shape[1:]))
        dist.reduce_scatter_tensor(out, g.contiguous(), group=ctx.group)
        return out, None, None


class _RS(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, group, n):
        ctx.group, ctx.n = group, n
        out = x.new_empty((x.shape[0] // n,) + tuple(x.shape[1:]))
        dist.reduce_scatter_tensor(out, x.contiguous(), group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = g.new_empty((g.shape[0] * ctx.n,) + tuple(g.shape[1:]))
        dist.all_gather_into_tensor(out, g.contiguous(), group=ctx.group)
        return out, None, None


def _p(shape, std, device, dtype, sharded=False):
    t = torch.empty(shape, device=device, dtype=dtype)
    with torch.no_grad():
        t.normal_(0.0, std)
    p = nn.Parameter(t)
    p.tp_sharded = sharded
    return p


def _ones(n, device, dtype):
    p = nn.Parameter(torch.ones(n, device=device, dtype=dtype))
    p.tp_sharded = False
    return p


def _q_rows(t: torch.Tensor):
    """e4m3 copy of t [R, C] with one fp32 scale per row (max|row| / 448)."""
    amax = t.abs().amax(-1, keepdim=True).float().clamp_min(1e-12)
    scale = amax / 448.0
    return (t.float() / scale).to(torch.float8_e4m3fn), scale


def _smm(a: torch.Tensor, b: torch.Tensor, out_dtype):
    """a [M, K] @ b[N, K]^T with row-wise e4m3 quantisation of both operands."""
    aq, sa = _q_rows(a)
    bq, sb = _q_rows(b)
    return torch._scaled_mm(aq, bq.t(), scale_a=sa, scale_b=sb.t(), out_dtype=out_dtype)


class _Fp8Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        return _smm(x, w, x.dtype)

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        return _smm(dy, w.t().contiguous(), dy.dtype), dy.t() @ x


def _linear(x, w, fp8: bool):
    return _Fp8Linear.apply(x, w) if fp8 else F.linear(x, w)


class _Block(nn.Module):
    def __init__(self, cfg: ModelConfig, n: int, device, dtype, fp8: bool = False):
        super().__init__()
        D, H, Hk, hd, Fd, s = cfg.d_model, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn_dim, cfg.init_std
        if H % n or Hk % n or Fd % n:
            raise ValueError("heads, kv heads and the ffn dim must divide by the tensor-parallel size")
        self.h, self.hk, self.hd, self.eps = H // n, Hk // n, hd, cfg.norm_eps
        self.fp8 = fp8
        self.n1 = _ones(D, device, dtype)
        self.wqkv = _p(((self.h + 2 * self.hk) * hd, D), s, device, dtype, True)
        self.wo = _p((D, self.h * hd), s, device, dtype, True)
        self.n2 = _ones(D, device, dtype)
        self.w13 = _p((2 * (Fd // n), D), s, device, dtype, True)
        self.w2 = _p((D, Fd // n), s, device, dtype, True)

    def forward(self, h, B, S, cos, sin, group, n):
        D = h.shape[-1]
        ag = (lambda t: _AG.apply(t, group, n)) if n > 1 else (lambda t: t)
        rs = (lambda t: _RS.apply(t, group, n)) if n > 1 else (lambda t: t)
        y = ag(F.rms_norm(h, (D,), self.n1, self.eps))
        T = y.shape[0]
        qkv = _linear(y, self.wqkv, self.fp8).view(T, self.h + 2 * self.hk, self.hd)
        qk = qkv[:, :self.h + self.hk]
        half = self.hd // 2
        q0, q1 = qk[..., :half], qk[..., half:]
        qk = torch.cat([q0 * cos - q1 * sin, q1 * cos + q0 * sin], dim=-1)
        q = qk[:, :self.h].view(B, S, self.h, self.hd).transpose(1, 2)
        k = qk[:, self.h:].view(B, S, self.hk, self.hd).transpose(1, 2)
        v = qkv[:, self.h + self.hk:].reshape(B, S, self.hk, self.hd).transpose(1, 2)
        o = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=self.hk != self.h)
        h = h + rs(_linear(o.transpose(1, 2).reshape(T, self.h * self.hd), self.wo, self.fp8))
        y = ag(F.rms_norm(h, (D,), self.n2, self.eps))
        g = _linear(y, self.w13, self.fp8)
        f = g.shape[-1] // 2
        return h + rs(_linear(F.silu(g[:, :f]) * g[:, f:], self.w2, self.fp8))


class TorchDenseTPLM(nn.Module):
    """Dense GQA LM (RMSNorm, RoPE, SwiGLU, untied head) with tensor + sequence parallelism."""

    def __init__(self, cfg: ModelConfig, device, group=None, dtype=torch.bfloat16, seed: int = 1234,
                 fp8: bool = False):
        super().__init__()
        torch.manual_seed(seed)
        if str(device).startswith("cuda"):
            torch.cuda.manual_seed(seed)
        self.cfg, self.group = cfg, group
        self.n = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        D, V = cfg.d_model, cfg.vocab_size
        self.embed = _p((V, D), cfg.init_std, device, dtype)
        self.blocks = nn.ModuleList([_Block(cfg, self.n, device, dtype, fp8) for _ in range(cfg.n_layers)])
        self.nf = _ones(D, device, dtype)
        self.head = _p((V, D), cfg.init_std, device, dtype)
        hd = cfg.head_dim
        inv = cfg.attn.rope_theta ** (-torch.arange(0, hd, 2, dtype=torch.float64) / hd)
        ang = torch.outer(torch.arange(cfg.max_seq_len, dtype=torch.float64) / cfg.attn.rope_scale, inv)
        self.register_buffer("cos", ang.cos().to(dtype).to(device), persistent=False)
        self.register_buffer("sin", ang.sin().to(dtype).to(device), persistent=False)

    def forward(self, ids, labels):
        B, S = ids.shape
        flat, lab = ids.reshape(-1), labels.reshape(-1)
        T = flat.numel()
        lo, hi = self.rank * T // self.n, (self.rank + 1) * T // self.n
        h = F.embedding(flat[lo:hi], self.embed)
        pos = torch.arange(S, device=ids.device).repeat(B)
        cos, sin = self.cos[pos][:, None], self.sin[pos][:, None]
        for blk in self.blocks:
            h = blk(h, B, S, cos, sin, self.group, self.n)
        y = F.rms_norm(h, (h.shape[-1],), self.nf, self.cfg.norm_eps)
        return F.cross_entropy(F.linear(y, self.head).float(), lab[lo:hi])


class TorchTPTrainer:
    """Gradient accumulation over micro-batches of one sequence, replicated-gradient all-reduce,
    global-norm clip, fused AdamW on fp32 masters."""

    def __init__(self, model: TorchDenseTPLM, tcfg: TrainConfig):
        self.model, self.tcfg, self.step_idx = model, tcfg, 0
        self.params = [p for p in model.parameters()]
        self.masters = [nn.Parameter(p.detach().float().clone()) for p in self.params]
        decay = [m for p, m in zip(self.params, self.masters) if p.dim() > 1]
        nodecay = [m for p, m in zip(self.params, self.masters) if p.dim() <= 1]
        self.opt = torch.optim.AdamW([{"params": decay, "weight_decay": tcfg.weight_decay},
                                      {"params": nodecay, "weight_decay": 0.0}], lr=tcfg.lr,
                                     betas=tuple(tcfg.betas), eps=tcfg.eps, fused=True)

    def step(self, ids, labels):
        from ..ops.optim import cosine_lr
        m, t = self.model, self.tcfg
        accum = max(1, t.grad_accum)
        total = None
        for ci, cl in zip(ids.chunk(accum), labels.chunk(accum)):
            loss = m(ci, cl) / accum
            loss.backward()
            total = loss.detach() if total is None else total + loss.detach()
        with torch.no_grad():
            rep = [p.grad for p in self.params if not p.tp_sharded and p.grad is not None]
            if m.n > 1 and rep:
                flat = torch.cat([g.reshape(-1) for g in rep])
                dist.all_reduce(flat, group=m.group)
                o = 0
                for g in rep:
                    g.copy_(flat[o:o + g.numel()].view_as(g))
                    o += g.numel()
            scale = 1.0 / m.n                       # every rank's loss is the mean over its tokens
            sh = torch.stack([p.grad.float().pow(2).sum() for p in self.params
                              if p.tp_sharded and p.grad is not None]).sum()
            if m.n > 1:
                dist.all_reduce(sh, group=m.group)
            sq = sh + torch.stack([g.float().pow(2).sum() for g in rep]).sum()
            coef = scale * (t.grad_clip / (sq.sqrt() * scale + 1e-6)).clamp(max=1.0) if t.grad_clip > 0 else scale
            for p, mst in zip(self.params, self.masters):
                mst.grad = None if p.grad is None else p.grad.float() * coef
                p.grad = None
            for gr in self.opt.param_groups:
                gr["lr"] = cosine_lr(self.step_idx, t.lr, t.warmup_steps, t.max_steps)
            self.opt.step()
            for p, mst in zip(self.params, self.masters):
                p.copy_(mst)
                mst.grad = None
        self.step_idx += 1
        if m.n > 1:
            dist.all_reduce(total, group=m.group)
            total = total / m.n
        return total
