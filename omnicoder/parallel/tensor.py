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
    """Tensor-parallel group.  transport "nccl": all_gather_into_tensor /
    reduce_scatter_tensor around plain GEMMs (and gloo on CPU).  transport
    "p2p" (CUDA): the fused collectives of this module over a symmetric
    peer-mapped arena -- the all-gather is done by the consuming GEMM's own
    loads (each rank's token shard is read tile by tile from its owner) and
    the reduce-scatter by the producing GEMM's epilogue (partial tiles stored
    into the row owner's staging slots, then summed locally)."""

    def __init__(self, group=None, transport: str = "nccl", arena_bytes: int = 64 << 20, fp8: bool = False):
        if fp8 and transport != "nccl":
            raise ValueError("fp8 tensor-parallel projections run with the nccl transport")
        self.fp8 = fp8                          # block-scaled fp8 fprop / dgrad GEMMs in the sharded projections
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.transport = transport
        self._arena_bytes = arena_bytes
        self.arena = None
        self._regions: dict = {}
        self._uses: dict = {}

    def shard(self, n: int, what: str) -> tuple[int, int]:
        if n % self.world:
            raise ValueError(f"{what} ({n}) must divide by the tensor-parallel size {self.world}")
        per = n // self.world
        return self.rank * per, (self.rank + 1) * per

    def copy_stream(self) -> "torch.cuda.Stream":
        if getattr(self, "_copy_stream", None) is None:
            self._copy_stream = torch.cuda.Stream()
        return self._copy_stream

    def fused(self, rows_local: int) -> bool:
        """Whether the fused peer-memory collectives apply to a shard of `rows_local` tokens."""
        return self.transport == "p2p" and self.world > 1 and rows_local % 128 == 0 and torch.cuda.is_available()

    def region(self, kind: str, nbytes: int):
        """An exchange region of at least `nbytes` per rank.  Two regions per kind alternate:
        a rank writes a region again only two collectives later, after the intervening
        collective's barrier, which every rank passes only once it has finished with the
        region (its copies and reductions precede that barrier in stream order) -- so one
        device barrier per collective suffices."""
        n = self._uses.get(kind, 0)
        self._uses[kind] = n + 1
        key = (kind, n & 1)
        r = self._regions.get(key)
        if r is None or r.nbytes[0] < nbytes:
            if self.arena is None:
                from .symm import SymmArena
                self.arena = SymmArena(self.group, torch.device("cuda", torch.cuda.current_device()),
                                       max(self._arena_bytes, 4 * nbytes))
            r = self.arena.alloc([nbytes] * self.world)
            self._regions[key] = r
        return r


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


# ----------------------------------------------------------------------------
# fused collectives over peer memory (transport "p2p")
# ----------------------------------------------------------------------------
_EPI_BF16, _EPI_SWIGLU = 0, 4


def _ag_gemm_fwd(x_local, w, tp, epi, H=None, b_mn=False, keep_full=False, swiglu_h=None):
    """gather(x_local over the group) @ w^T.  Remote data read over NVLink is not cached in
    this GPU's L2, so each peer shard crosses the link once: copy engines bring the shards
    into a local buffer in ring order (on a side stream) while the GEMM runs on the rows
    already present, starting with this rank's own shard.  Returns (out, gathered input)."""
    from ..ops import _ext
    C = _ext.load()
    rows, D = x_local.shape
    nbytes = rows * D * 2
    reg = tp.region("ag", nbytes)
    reg.view(torch.bfloat16, rows, D).copy_(x_local)
    tp.arena.barrier()                          # every rank's shard is in place
    N = w.shape[1] if b_mn else w.shape[0]
    ncol = N // 2 if epi == _EPI_SWIGLU else (2 * N if swiglu_h is not None else N)
    dev = x_local.device
    out = torch.empty(tp.world * rows, ncol, device=dev, dtype=torch.bfloat16)
    full = torch.empty(tp.world * rows, D, device=dev, dtype=torch.bfloat16)
    main = torch.cuda.current_stream(dev)
    side = tp.copy_stream()
    side.wait_stream(main)
    events = {}
    with torch.cuda.stream(side):
        full[tp.rank * rows:(tp.rank + 1) * rows].copy_(x_local)
        for j in range(1, tp.world):
            r = (tp.rank + j) % tp.world
            C.peer_copy(full[r * rows:(r + 1) * rows], reg.ptrs[r], nbytes)
            ev = torch.cuda.Event()
            ev.record(side)
            events[r] = ev
    # GEMM launches over ring-contiguous groups of shards: this rank's own shard (no copy to wait
    # for), then the nearest peers, then the rest (fewer, larger launches than one per shard)
    def run(r0, nr):
        if r0 + nr <= tp.world:
            spans = [(r0, nr)]
        else:
            spans = [(r0, tp.world - r0), (0, r0 + nr - tp.world)]
        for a, n in spans:
            lo, hi = a * rows, (a + n) * rows
            src = x_local if (n == 1 and a == tp.rank) else full[lo:hi]
            h = None if H is None else H[lo:hi]
            rr = None if swiglu_h is None else swiglu_h[lo:hi]
            C.gemm(src, w, out[lo:hi], False, b_mn, epi, 1.0, rr, h, 256)

    run(tp.rank, 1)
    rest = tp.world - 1
    first = max(1, rest // 3)
    groups = [(1, first), (1 + first, rest - first)] if rest > 1 else ([(1, 1)] if rest == 1 else [])
    for j0, n in groups:
        if n <= 0:
            continue
        for j in range(j0, j0 + n):
            main.wait_event(events[(tp.rank + j) % tp.world])
        run((tp.rank + j0) % tp.world, n)
    main.wait_stream(side)
    # the side stream's copies read `full`/`x_local` allocations that the caching allocator
    # must not recycle before they finish
    full.record_stream(side)
    x_local.record_stream(side)
    return out, (full if keep_full else None)


def _gemm_rs_fwd(x_full, w, tp, residual=None, b_mn=False):
    """Partial products x_full @ w^T reduce-scattered over the group: the GEMM stores every
    tile into its row owner's staging slot, the owner sums the slots (+ residual)."""
    from ..ops import _ext
    C = _ext.load()
    T, _ = x_full.shape
    rows = T // tp.world
    N = w.shape[1] if b_mn else w.shape[0]
    reg = tp.region("rs", tp.world * rows * N * 2)
    C.gemm_rs(x_full.contiguous(), w, reg.ptrs, rows, N, tp.rank, b_mn)
    tp.arena.barrier()                          # every partial tile has landed
    out = torch.empty(rows, N, device=x_full.device, dtype=torch.bfloat16)
    C.tp_reduce(reg.view(torch.bfloat16, tp.world, rows, N), out,
                None if residual is None else residual.contiguous())
    return out


class _AGLinear(torch.autograd.Function):
    """y [T, N_shard] = gather(x_local) @ w^T (column-parallel projection)."""

    @staticmethod
    def forward(ctx, x_local, w, tp):
        ctx.tp = tp
        out, full = _ag_gemm_fwd(x_local, w, tp, _EPI_BF16, keep_full=True)
        ctx.save_for_backward(full, w)
        return out

    @staticmethod
    def backward(ctx, dy):
        from ..ops.gemm import mm_tn
        full, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = _gemm_rs_fwd(dy, w, ctx.tp, b_mn=True)        # reduce-scatter(dy @ w) in the GEMM epilogue
        return dx, mm_tn(dy, full), None


class _TPSwiGLUMLP(torch.autograd.Function):
    """Sequence-parallel SwiGLU MLP block: y_local = RS(silu(g) * u @ w2^T) + residual with
    [g | u] = gather(x_local) @ w13^T."""

    @staticmethod
    def forward(ctx, x_local, w13, w2, residual, tp):
        T = x_local.shape[0] * tp.world
        H = torch.empty(T, w13.shape[0], device=x_local.device, dtype=torch.bfloat16)
        act, full = _ag_gemm_fwd(x_local, w13, tp, _EPI_SWIGLU, H=H, keep_full=True)
        y = _gemm_rs_fwd(act, w2, tp, residual)
        ctx.tp = tp
        ctx.has_res = residual is not None
        ctx.save_for_backward(full, w13, w2, H, act)
        return y

    @staticmethod
    def backward(ctx, dy):
        from ..ops.gemm import EPI_SWIGLU_BWD, mm_tn
        full, w13, w2, H, act = ctx.saved_tensors
        tp = ctx.tp
        dy = dy.contiguous()
        # dH = (gather(dy) @ w2) through the SwiGLU backward epilogue, gather staged like forward
        dH, dy_full = _ag_gemm_fwd(dy, w2, tp, EPI_SWIGLU_BWD, H=None, b_mn=True, keep_full=True,
                                   swiglu_h=H)
        dw2 = mm_tn(dy_full, act)
        dx = _gemm_rs_fwd(dH, w13, tp, b_mn=True)
        dw13 = mm_tn(dH, full)
        return dx, dw13, dw2, (dy if ctx.has_res else None), None


class _LinearRS(torch.autograd.Function):
    """y_local = reduce-scatter(x_full @ w^T) (+ residual) (row-parallel projection)."""

    @staticmethod
    def forward(ctx, x_full, w, residual, tp):
        ctx.tp = tp
        ctx.has_res = residual is not None
        ctx.save_for_backward(x_full, w)
        return _gemm_rs_fwd(x_full, w, tp, residual)

    @staticmethod
    def backward(ctx, dy):
        from ..ops.gemm import mm_tn
        x_full, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx, dy_full = _ag_gemm_fwd(dy, w, ctx.tp, _EPI_BF16, b_mn=True, keep_full=True)
        return dx, mm_tn(dy_full, x_full), (dy if ctx.has_res else None), None


def tp_linear_ag(x_local: torch.Tensor, w: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """Column-parallel projection of the sequence-sharded input: gather over the group, @ w^T."""
    if tp.fused(x_local.shape[0]):
        return _AGLinear.apply(x_local, w, tp)
    from ..ops.layers import linear
    return linear(all_gather_seq(x_local, tp), w)


def tp_swiglu_mlp(x_local: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, tp: TPContext,
                  residual: torch.Tensor | None = None) -> torch.Tensor:
    """Sequence-parallel SwiGLU MLP block (w13: this rank's gate|up rows, w2: its down columns)."""
    if tp.fused(x_local.shape[0]):
        return _TPSwiGLUMLP.apply(x_local, w13, w2, residual, tp)
    from ..ops.layers import swiglu_mlp
    y = reduce_scatter_seq(swiglu_mlp(all_gather_seq(x_local, tp), w13, w2), tp)
    return y if residual is None else y + residual


def tp_linear_rs(x_full: torch.Tensor, w: torch.Tensor, tp: TPContext,
                 residual: torch.Tensor | None = None) -> torch.Tensor:
    """Row-parallel projection: partial x_full @ w^T reduce-scattered over the group (+ residual)."""
    if tp.fused(x_full.shape[0] // tp.world):
        return _LinearRS.apply(x_full, w, residual, tp)
    from ..ops.layers import linear
    y = reduce_scatter_seq(linear(x_full, w), tp)
    return y if residual is None else y + residual


def scatter_seq(x: torch.Tensor, tp: TPContext) -> torch.Tensor:
    """This rank's token shard of a replicated [T, ...] tensor (no communication)."""
    lo, hi = tp.shard(x.shape[0], "token count")
    return x[lo:hi]


class TensorParallel:
    """Trainer-facing layout object: optimizer over local parameters, gradient
    all-reduce of the replicated ones over the TP group (bucketed, one NCCL call
    per bucket)."""

    def __init__(self, group=None, bucket_bytes: int = 64 << 20, transport: str = "nccl", fp8: bool = False):
        self.tp = TPContext(group, transport=transport, fp8=fp8)
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
