"""Expert parallelism: routed experts sharded over the ranks of a group.

Rank r owns experts [r * El, (r + 1) * El) (El = E / world).  Each rank routes
its own tokens; every (token, k) pair travels to the owner of its expert,
is processed by the owner's grouped SwiGLU GEMMs and travels back to be
combined with the routing weight.

Receive layout (identical on every rank, computed from the all-gathered
per-(source, expert) counts C[s, e]):
  owner r holds its El experts back to back; expert e's segment holds the
  kept rows of source 0, then source 1, ... in token order, padded to a
  multiple of 128 rows (the grouped tcgen05 GEMM's tile height).
With a capacity (tokens per expert, over the whole group) the first
`capacity` pairs of each expert in (source rank, token) order are kept --
the same pairs a single process keeps for the concatenated batch.

Two transports implement the same layout:
  * "p2p" (CUDA): the sm_100a kernels of ep_comm.cu over a symmetric
    peer-mapped arena: dispatch fused with the permutation (peer stores),
    combine fused with the weighted sum (peer loads), owner-side routing-weight
    gradient, device barriers with bounded waits.
  * "nccl" / CPU: torch.distributed.all_to_all_single with plain PyTorch
    expert math (torch._grouped_mm over the local experts, a batched weighted
    sum) -- the NCCL + cuBLAS comparison path on GPUs and the gloo path of the
    CPU tests.

The reference has no expert parallelism (its EP launcher only sets an
environment variable that the MoE layer in use never reads:
src/omnicoder/tools/torchrun_ep.py:36-38, src/omnicoder/modeling/moe_layer.py).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..ops import _ext
from ..ops.gemm import EPI_BF16, EPI_SWIGLU, EPI_SWIGLU_BWD, deinterleave_cols, mm_nn, mm_nt, mm_tn
from ..ops.moe import cap_rows_for, route_torch


# ----------------------------------------------------------------------------
# Layout (host, numpy): identical on every rank
# ----------------------------------------------------------------------------
@dataclass
class EPLayout:
    kept: np.ndarray          # [N, E] rows of source s kept for expert e
    dst_base: np.ndarray      # [E] first row of this rank's pairs inside expert e's segment (on its owner)
    keep_lim: np.ndarray      # [E] pairs of this rank kept per expert
    offs_local: np.ndarray    # [El + 1] padded segment offsets of this rank's receive buffer
    kept_local: np.ndarray    # [El] rows (before padding) of each local expert
    rows: list                # [N] padded receive rows of every rank
    pairs: list               # [N] T_s * K of every rank (size of its routing-weight gradient)


def ep_layout(C: np.ndarray, me: int, El: int, capacity: int = 0) -> EPLayout:
    C = np.asarray(C, dtype=np.int64)
    N, E = C.shape
    before = np.cumsum(C, axis=0) - C                         # rows of earlier sources, per expert
    if capacity > 0:
        kept = np.clip(np.minimum(C, capacity - before), 0, None)
    else:
        kept = C.copy()
    seg = kept.sum(0)                                         # [E]
    seg_pad = ((seg + 127) // 128 * 128).reshape(N, El)
    seg_base = (np.cumsum(seg_pad, axis=1) - seg_pad).reshape(E)
    kept_before = np.cumsum(kept, axis=0) - kept
    dst_base = seg_base + kept_before[me]
    offs_local = np.concatenate([[0], np.cumsum(seg_pad[me])])
    return EPLayout(kept=kept, dst_base=dst_base, keep_lim=kept[me].copy(), offs_local=offs_local,
                    kept_local=seg.reshape(N, El)[me].copy(), rows=[int(x) for x in seg_pad.sum(1)],
                    pairs=[int(x) for x in C.sum(1)])


def local_ranks(idx: torch.Tensor, E: int) -> torch.Tensor:
    """Rank of each (token, k) pair among this rank's pairs of the same expert, in token order."""
    flat = idx.reshape(-1).long()
    onehot = F.one_hot(flat, E)
    return (onehot.cumsum(0) - 1).gather(1, flat.unsqueeze(1)).squeeze(1).view_as(idx)


# ----------------------------------------------------------------------------
# Context
# ----------------------------------------------------------------------------
class EPContext:
    """Expert-parallel group of one process: rank, world, transport, arena."""

    def __init__(self, group=None, transport: str = "auto", device=None, arena_bytes: int = 1 << 30,
                 layout: str = "device", buffer_factor: float = 2.0, epilogue_push: bool = True,
                 gate_tiles: bool = False):
        """layout (p2p transport): "device" -- routing counts are exchanged and the receive
        layout is computed on the device; every MoE layer has fixed slabs of
        El * seg_cap rows per rank (seg_cap = the capacity, or, dropless, buffer_factor x the
        balanced per-expert load, rounded up to 128), so nothing reaches the host and the
        step can be captured as a CUDA graph.  Nothing is dropped while an owner's routed
        rows fit its slab; when they do not, each of its experts keeps at most seg_cap rows
        (the pairs lost are counted in `dropped_pairs()`).  "host" -- counts are all-gathered
        to the host once per layer and the slabs are sized exactly (no drop beyond the
        capacity).  epilogue_push (device layout, bf16 experts): the expert GEMMs' epilogues
        store their output rows into the sources' (token, k) slots; False: the rows are
        written locally and returned by a copy kernel afterwards.  gate_tiles (device layout,
        bf16 experts): instead of a barrier after the dispatch (and after the backward's
        gradient push), each source signals once its rows are out and the grouped GEMM starts a
        tile as soon as the sources of its rows have signalled."""
        if layout not in ("device", "host"):
            raise ValueError(f"unknown expert-parallel layout {layout!r}")
        self.layout = layout
        self.buffer_factor = float(buffer_factor)
        self.epilogue_push = bool(epilogue_push)
        self.gate_tiles = bool(gate_tiles)
        self.group = group if group is not None else dist.group.WORLD
        self.rank = dist.get_rank(self.group)
        self.world = dist.get_world_size(self.group)
        self.device = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
        if transport == "auto":
            transport = "p2p" if self.device.type == "cuda" else "nccl"
        self.transport = transport
        self.arena = None
        self._arena_bytes = arena_bytes
        self.stats = {"host_syncs": 0}
        self._plans: dict = {}           # device layout, per (tokens per rank, training?): fixed slabs
        self._cursor = 0
        self._dropped = None
        # id(bf16 expert weight) -> (e4m3 weight, fp32 128x128 block scales): when both expert
        # weights of a layer are present, its forward expert GEMMs run in block-scaled fp8
        self.fp8_weights: dict = {}

    def set_fp8_weights(self, w13: torch.Tensor, w2: torch.Tensor):
        """Quantise a layer's expert weight stacks (w13 [El, 2F, D], w2 [El, D, F], bf16) for the
        fp8 path (call again after every optimiser step): the forward GEMMs use them as they are,
        the input-gradient GEMM through the gate|up experts w13's transpose (key ("t", id))."""
        from ..ops.fp8 import quantize_weight
        for w in (w13, w2):
            self.fp8_weights[id(w)] = quantize_weight(w.detach())
        if w13.shape[-1] % 128 == 0 and w13.shape[-2] % 128 == 0:
            self.fp8_weights[("t", id(w13))] = quantize_weight(w13.detach().transpose(-1, -2).contiguous())

    def experts_of(self, E: int) -> tuple[int, int]:
        if E % self.world:
            raise ValueError(f"{E} experts do not divide over {self.world} expert-parallel ranks")
        El = E // self.world
        return self.rank * El, (self.rank + 1) * El

    def ensure_arena(self):
        if self.arena is None:
            from .symm import SymmArena
            self.arena = SymmArena(self.group, self.device, self._arena_bytes)
        return self.arena

    def begin_step(self):
        """Start of a micro-step.  Host layout: every rank has finished reading the previous
        step's regions (device barrier) before they are handed out again.  Device layout:
        the k-th MoE layer of every step reuses the k-th set of slabs; the barriers inside
        each layer's exchange already order every reuse, so nothing is launched here."""
        if self.layout == "device" and self.transport == "p2p":
            self._cursor = 0
            return
        if self.arena is not None:
            self.arena.barrier()
            self.arena.reset()

    def dropped_pairs(self) -> int:
        """(token, expert) pairs of this rank dropped by the device layout's slab bound so far
        (reads the device counter: a host sync; call it outside timed loops)."""
        return 0 if self._dropped is None else int(self._dropped.item())

    # ---- device layout: fixed slabs ----------------------------------------------------
    def seg_cap(self, T: int, k: int, E: int, capacity: int) -> int:
        if capacity > 0:
            return (capacity + 127) // 128 * 128
        bal = math.ceil(self.buffer_factor * self.world * T * k / E)
        return max(128, (bal + 127) // 128 * 128)

    def slot(self, T: int, k: int, E: int, El: int, D: int, capacity: int, train: bool):
        """(slabs of the next MoE layer, shared slabs) for T tokens per rank.  With autograd
        recording, every MoE layer of a step has its own slabs (its forward's slabs are read by
        its backward) and the cursor advances; without (inference), one set serves every layer
        (each layer's barriers order the reuse).  Slabs are allocated on first use; every rank
        allocates the same sizes in the same order, and every rank must pass the same T (checked
        once per T with one collective).  `train` must be decided outside autograd.Function.forward,
        where grad mode is always off."""
        key = (T, train)
        plan = self._plans.get(key)
        if plan is None:
            t = torch.tensor([T], device=self.device)
            mx, mn = t.clone(), t.clone()
            dist.all_reduce(mx, op=dist.ReduceOp.MAX, group=self.group)
            dist.all_reduce(mn, op=dist.ReduceOp.MIN, group=self.group)
            if int(mx.item()) != int(mn.item()):
                raise ValueError("the device expert-parallel layout needs the same token count on every rank")
            if self._dropped is None:
                self._dropped = torch.zeros(1, dtype=torch.int32, device=self.device)
            plan = self._plans[key] = {"slots": [], "shared": None}
        arena = self.ensure_arena()
        cap = self.seg_cap(T, k, E, capacity)
        R = El * cap
        N = self.world
        if plan["shared"] is None:
            plan["shared"] = _Shared(arena, N, R, D, T * k, E, backward=train)
        i = self._cursor if train else 0
        if i == len(plan["slots"]):
            plan["slots"].append(_Slot(arena, N, R, D, E, El, cap, self.device, T * k))
        sl = plan["slots"][i]
        if (sl.R, sl.D, sl.E, sl.cap, sl.pairs) != (R, D, E, cap, T * k):
            raise ValueError("MoE layers of one step changed shape between steps")
        if train:
            self._cursor += 1
        return sl, plan["shared"]

    def all_gather_counts(self, counts: torch.Tensor) -> np.ndarray:
        """[E] int32 per rank -> host [N, E] (one small collective + one host sync)."""
        out = [torch.empty_like(counts) for _ in range(self.world)]
        dist.all_gather(out, counts.contiguous(), group=self.group)
        self.stats["host_syncs"] += 1
        return torch.stack(out).cpu().numpy()


class _Slot:
    """Fixed peer-mapped slabs of one MoE layer (device layout): receive rows x and their routing
    metadata (owner side), the (token, k) slots ys that the owners' down-projection epilogues
    push the expert outputs into (source side); plus this rank's device-computed layout."""

    def __init__(self, arena, N, R, D, E, El, cap, device, pairs):
        self.R, self.D, self.E, self.cap, self.pairs = R, D, E, cap, pairs
        self.x = arena.alloc([R * D * 2] * N)
        self.meta = arena.alloc([R * 16] * N)
        self.ys = arena.alloc([pairs * D * 2] * N)
        z = lambda n: torch.zeros(n, dtype=torch.int32, device=device)
        self.dst_base, self.keep_lim, self.offs_local, self.kept_local = z(E), z(E), z(El + 1), z(El)
        self.src_pref = z(El * (N + 1))     # row offset of each source inside each local expert segment
        self.rows = [R] * N


class _Shared:
    """Slabs shared by every MoE layer (device layout): the count board and, when training,
    the backward's weighted output gradients pushed to the owners (receive rows) and the input
    gradients that the owners' epilogues push back into the sources' (token, k) slots."""

    def __init__(self, arena, N, R, D, pairs, E, backward: bool = True):
        self.board = arena.alloc([N * E * 4] * N)
        # per-source readiness flags (one-way signals after a source's stores into this rank's
        # receive rows) and this rank's signal counter; zeroed on every rank before first use
        self.ready = arena.alloc([max(16, N * 4)] * N)
        self.ready.view(torch.int32, max(4, N)).zero_()
        self.sig_ctr = torch.zeros(1, dtype=torch.int32, device=self.ready.local.device)
        arena.barrier()
        self.dy = self.dxs = None
        if backward:
            self.dy = arena.alloc([R * D * 2] * N)
            self.dxs = arena.alloc([pairs * D * 2] * N)
        self.pairs = [pairs] * N


# ----------------------------------------------------------------------------
# p2p transport (CUDA, fused kernels over the symmetric arena)
# ----------------------------------------------------------------------------
def _i32(dev, *arrays) -> list[torch.Tensor]:
    """Upload int32 arrays with one host->device copy."""
    flat = np.concatenate([np.asarray(a, dtype=np.int32).ravel() for a in arrays])
    t = torch.from_numpy(flat).pin_memory().to(dev, non_blocking=True)
    out, o = [], 0
    for a in arrays:
        n = int(np.asarray(a).size)
        out.append(t[o:o + n])
        o += n
    return out


class _EPMoEP2P(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, router_w, w13, w2, add, ep, k, capacity, renorm, aux_alpha, z_beta, gs):
        C = _ext.load()
        arena = ep.ensure_arena()
        x = x.contiguous()
        T, D = x.shape
        E = router_w.shape[0]
        El = w13.shape[0]
        F2 = w13.shape[1]
        me = ep.rank
        logits = mm_nt(x, router_w, out_f32=True)
        idx, wts, probs = C.router_topk(logits, k, renorm)
        counts, loc_off, pos, _ = C.moe_plan(idx, E, 0, cap_rows_for(T, k, E, 0))
        lay = ep_layout(ep.all_gather_counts(counts), me, El, capacity)
        rows = [max(r, 128) for r in lay.rows]
        dst_base, keep_lim, offs_local, kept_local = _i32(x.device, lay.dst_base, lay.keep_lim, lay.offs_local,
                                                           lay.kept_local)
        rx = arena.alloc([r * D * 2 for r in rows])
        rmeta = arena.alloc([r * 16 for r in rows])
        slot = C.ep_dispatch(x, idx, pos, loc_off, dst_base, keep_lim, wts, rx.ptrs, rmeta.ptrs, rows, El, me)
        R = rows[me]
        x_recv = rx.view(torch.bfloat16, R, D)
        meta = rmeta.view(torch.int32, R, 4)
        C.ep_pad_rows(x_recv, meta, offs_local, kept_local)
        arena.barrier()                                       # all pairs have landed
        ry = arena.alloc([r * D * 2 for r in rows])
        y_recv = ry.view(torch.bfloat16, R, D)
        q13 = ep.fp8_weights.get(id(w13)) if ep.fp8_weights else None
        q2 = ep.fp8_weights.get(id(w2)) if ep.fp8_weights else None
        if q13 is not None and q2 is not None:
            # block-scaled fp8 expert GEMMs (weights quantised once per optimiser step by the
            # caller; activations per 1 x 128 block here); backward uses the bf16 weights
            from ..ops.fp8 import fp8_grouped_swiglu
            # SwiGLU and the requantisation of its output run in the gate|up GEMM's epilogue
            H, act, aq, sa = fp8_grouped_swiglu(x_recv, q13[0], q13[1], offs_local, R)
            C.fp8_gemm(aq, sa, q2[0], q2[1].reshape(-1), y_recv, offs_local, R)
        else:
            act = torch.empty(R, F2 // 2, device=x.device, dtype=torch.bfloat16)
            H = torch.empty(R, F2, device=x.device, dtype=torch.bfloat16)
            C.gemm_grouped_m(x_recv, w13, offs_local, act, False, EPI_SWIGLU, 1.0, None, H, 256, R)
            C.gemm_grouped_m(act, w2, offs_local, y_recv, False, EPI_BF16, 1.0, None, None, 256, R)
        arena.barrier()                                       # every owner's outputs are ready
        out = C.ep_combine(slot, idx, wts, ry.ptrs, rows, El, D, None if add is None else add.contiguous())
        ctx.save_for_backward(x, router_w, w13, w2, logits, probs, idx, wts, counts, slot, offs_local, kept_local,
                              H, act)
        # arena regions are views of one shared buffer (one autograd version counter for all
        # of them), so they are kept on ctx instead of going through save_for_backward; the
        # arena is not recycled before this backward has run (reset at the next micro-step)
        ctx.x_recv, ctx.meta, ctx.y_recv = x_recv, meta, y_recv
        ctx.ep, ctx.ry, ctx.rows, ctx.lay = ep, ry, rows, lay
        ctx.cfg = (k, renorm, aux_alpha, z_beta, gs, add is not None)
        aux = x.new_zeros((), dtype=torch.float32)
        if aux_alpha > 0:
            aux = aux + aux_alpha * E * ((counts.float() / (T * k)) * probs.mean(0)).sum()
        if z_beta > 0:
            lse = torch.logsumexp(logits, dim=-1)
            aux = aux + z_beta * (lse * lse).mean()
        ctx.mark_non_differentiable(aux)
        return out, aux

    @staticmethod
    def backward(ctx, dout, daux):
        (x, router_w, w13, w2, logits, probs, idx, wts, counts, slot, offs_local, kept_local, H,
         act) = ctx.saved_tensors
        x_recv, meta, y_recv = ctx.x_recv, ctx.meta, ctx.y_recv
        k, renorm, aux_alpha, z_beta, gs, has_add = ctx.cfg
        ep, rows, lay = ctx.ep, ctx.rows, ctx.lay
        arena = ep.arena
        C = _ext.load()
        T, D = x.shape
        El = w13.shape[0]
        R = rows[ep.rank]
        dout = dout.contiguous()
        rdy = arena.alloc([r * D * 2 for r in rows])
        rdw = arena.alloc([max(p, 1) * 4 for p in lay.pairs])
        dwts = rdw.view(torch.float32, T, k)
        dwts.zero_()                                          # dropped pairs keep a zero gradient
        C.ep_push(dout, slot, idx, rdy.ptrs, rows, El)
        arena.barrier()                                       # all output gradients have landed
        dy_recv = rdy.view(torch.bfloat16, R, D)
        C.ep_owner_bwd(dy_recv, y_recv, meta, offs_local, kept_local, rdw.ptrs, [max(p, 1) for p in lay.pairs])
        dH = torch.empty_like(H)
        C.gemm_grouped_m(dy_recv, w2, offs_local, dH, True, EPI_SWIGLU_BWD, 1.0, H, None, 256, R)
        dw2 = torch.empty_like(w2)
        C.gemm_grouped_k(dy_recv, act, offs_local, dw2, EPI_BF16, 1.0, 256)
        rdx = arena.alloc([r * D * 2 for r in rows])
        dx_recv = rdx.view(torch.bfloat16, R, D)
        C.gemm_grouped_m(dH, w13, offs_local, dx_recv, True, EPI_BF16, 1.0, None, None, 256, R)
        dw13 = torch.empty_like(w13)
        C.gemm_grouped_k(dH, x_recv, offs_local, dw13, EPI_BF16, 1.0, 256)
        arena.barrier()                                       # input gradients and weight gradients are ready
        dlogits, _ = C.router_bwd(logits, probs, idx, dwts, counts, renorm, aux_alpha * gs, z_beta * gs)
        dx_router = mm_nn(dlogits, router_w)
        dx = C.ep_combine(slot, idx, None, rdx.ptrs, rows, El, D, dx_router)
        drouter = mm_tn(dlogits, x)
        return (dx, drouter, dw13, dw2, (dout if has_add else None), None, None, None, None, None, None, None)


class _EPMoEDev(torch.autograd.Function):
    """p2p transport with the device-computed layout: no host synchronisation anywhere in the
    layer (forward or backward), fixed slabs, device-epoch barriers -- capturable in a CUDA graph."""

    @staticmethod
    def forward(ctx, x, router_w, w13, w2, add, ep, k, capacity, renorm, aux_alpha, z_beta, gs, train):
        C = _ext.load()
        x = x.contiguous()
        T, D = x.shape
        E = router_w.shape[0]
        El = w13.shape[0]
        F2 = w13.shape[1]
        me = ep.rank
        sl, sh = ep.slot(T, k, E, El, D, capacity, train)
        arena = ep.arena
        R = sl.R
        logits = mm_nt(x, router_w, out_f32=True)
        idx, wts, probs = C.router_topk(logits, k, renorm)
        counts, loc_off, pos, _ = C.moe_plan(idx, E, 0, cap_rows_for(T, k, E, 0))
        # counts -> every rank's board, device barrier, layout from the board
        C.ep_exchange_layout(counts, sh.board.ptrs, arena.sig_ptrs, me, arena.epoch_ctr, El, capacity, sl.cap,
                             sl.dst_base, sl.keep_lim, sl.offs_local, sl.kept_local, ep._dropped, sl.src_pref)
        slot = C.ep_dispatch(x, idx, pos, loc_off, sl.dst_base, sl.keep_lim, wts, sl.x.ptrs, sl.meta.ptrs, sl.rows,
                             El, me)
        x_recv = sl.x.view(torch.bfloat16, R, D)
        meta = sl.meta.view(torch.int32, R, 4)
        C.ep_pad_rows(x_recv, meta, sl.offs_local, sl.kept_local)
        offs_local = sl.offs_local
        q13 = ep.fp8_weights.get(id(w13)) if ep.fp8_weights else None
        q2 = ep.fp8_weights.get(id(w2)) if ep.fp8_weights else None
        gate = {}
        if (q13 is not None and q2 is not None) or not ep.gate_tiles:
            arena.barrier()                                   # all pairs have landed
        else:
            # one-way signal; the gate|up GEMM starts each tile once the sources of its rows have signalled
            C.ep_signal(sh.ready.ptrs, me, sh.sig_ctr)
            gate = dict(ready_ptr=sh.ready.ptrs[me], ready_epoch=sh.sig_ctr, src_pref=sl.src_pref, nsrc=ep.world,
                        me=me)
        # the down projection's epilogue stores every output row into its source's (token, k)
        # slot (over NVLink for peers), so the combine transfer overlaps the GEMM (the block-scaled
        # GEMM writes its rows locally and ep_return_rows sends them)
        if q13 is not None and q2 is not None:
            from ..ops.fp8 import fp8_grouped_swiglu
            # SwiGLU and the requantisation of its output run in the gate|up GEMM's epilogue
            H, act, aq, sa = fp8_grouped_swiglu(x_recv, q13[0], q13[1], offs_local, R)
            y_loc = torch.empty(R, D, device=x.device, dtype=torch.bfloat16)
            C.fp8_gemm(aq, sa, q2[0], q2[1].reshape(-1), y_loc, offs_local, R)
            C.ep_return_rows(y_loc, meta, offs_local, sl.ys.ptrs, [T * k] * ep.world)
        else:
            act = torch.empty(R, F2 // 2, device=x.device, dtype=torch.bfloat16)
            H = torch.empty(R, F2, device=x.device, dtype=torch.bfloat16)
            C.gemm_grouped_m(x_recv, w13, offs_local, act, False, EPI_SWIGLU, 1.0, None, H, 256, R, **gate)
            if ep.epilogue_push:
                C.gemm_grouped_m_push(act, w2, offs_local, meta, sl.ys.ptrs, T * k, False, R)
            else:
                y_loc = torch.empty(R, D, device=x.device, dtype=torch.bfloat16)
                C.gemm_grouped_m(act, w2, offs_local, y_loc, False, EPI_BF16, 1.0, None, None, 256, R)
                C.ep_return_rows(y_loc, meta, offs_local, sl.ys.ptrs, [T * k] * ep.world)
        arena.barrier()                                       # every owner has pushed its outputs
        ys = sl.ys.view(torch.bfloat16, T * k, D)
        out = C.ep_combine_local(slot, ys, wts, None if add is None else add.contiguous())
        ctx.save_for_backward(x, router_w, w13, w2, logits, probs, idx, wts, counts, slot, H, act)
        # the slabs are views of the shared arena (kept on ctx, not saved tensors); the next
        # forward of this layer rewrites them only after this backward
        ctx.ep, ctx.sl, ctx.sh = ep, sl, sh
        ctx.cfg = (k, renorm, aux_alpha, z_beta, gs, add is not None)
        aux = x.new_zeros((), dtype=torch.float32)
        if aux_alpha > 0:
            aux = aux + aux_alpha * E * ((counts.float() / (T * k)) * probs.mean(0)).sum()
        if z_beta > 0:
            lse = torch.logsumexp(logits, dim=-1)
            aux = aux + z_beta * (lse * lse).mean()
        ctx.mark_non_differentiable(aux)
        return out, aux

    @staticmethod
    def backward(ctx, dout, daux):
        x, router_w, w13, w2, logits, probs, idx, wts, counts, slot, H, act = ctx.saved_tensors
        k, renorm, aux_alpha, z_beta, gs, has_add = ctx.cfg
        ep, sl, sh = ctx.ep, ctx.sl, ctx.sh
        arena = ep.arena
        C = _ext.load()
        T, D = x.shape
        El = w13.shape[0]
        R = sl.R
        x_recv = sl.x.view(torch.bfloat16, R, D)
        meta = sl.meta.view(torch.int32, R, 4)
        ys = sl.ys.view(torch.bfloat16, T * k, D)
        dout = dout.contiguous()
        # routing-weight gradients from the pushed outputs (local), weighted output gradients
        # pushed to the owners' receive rows
        dwts = torch.empty(T, k, device=x.device, dtype=torch.float32)
        C.ep_source_bwd(dout, ys, slot, idx, wts, dwts, sh.dy.ptrs, sl.rows, El)
        gate = {}
        if ep.gate_tiles:
            C.ep_signal(sh.ready.ptrs, ep.rank, sh.sig_ctr)  # this rank's output gradients are out
            # each tile of the dact GEMM starts once the sources of its rows have signalled
            gate = dict(ready_ptr=sh.ready.ptrs[ep.rank], ready_epoch=sh.sig_ctr, src_pref=sl.src_pref,
                        nsrc=ep.world, me=ep.rank)
        else:
            arena.barrier()                                   # all output gradients have landed
        dy_recv = sh.dy.view(torch.bfloat16, R, D)
        C.ep_pad_rows(dy_recv, None, sl.offs_local, sl.kept_local)
        dH = torch.empty_like(H)
        C.gemm_grouped_m(dy_recv, w2, sl.offs_local, dH, True, EPI_SWIGLU_BWD, 1.0, H, None, 256, R, **gate)
        dw2 = torch.empty_like(w2)
        C.gemm_grouped_k(dy_recv, act, sl.offs_local, dw2, EPI_BF16, 1.0, 256)
        q13t = ep.fp8_weights.get(("t", id(w13))) if ep.fp8_weights else None
        # input gradients pushed by the epilogue into the sources' (token, k) slots
        if q13t is not None:
            # fp8 input gradient through the gate|up experts (dH per 1 x 128 block, w13^T blocks)
            from ..ops.fp8 import quantize_act
            dq, sdq = quantize_act(dH, offsets=sl.offs_local)
            dx_loc = torch.empty(R, D, device=x.device, dtype=torch.bfloat16)
            C.fp8_gemm(dq, sdq, q13t[0], q13t[1].reshape(-1), dx_loc, sl.offs_local, R)
            C.ep_return_rows(dx_loc, meta, sl.offs_local, sh.dxs.ptrs, [T * k] * ep.world)
        elif ep.epilogue_push:
            C.gemm_grouped_m_push(dH, w13, sl.offs_local, meta, sh.dxs.ptrs, T * k, True, R)
        else:
            dx_loc = torch.empty(R, D, device=x.device, dtype=torch.bfloat16)
            C.gemm_grouped_m(dH, w13, sl.offs_local, dx_loc, True, EPI_BF16, 1.0, None, None, 256, R)
            C.ep_return_rows(dx_loc, meta, sl.offs_local, sh.dxs.ptrs, [T * k] * ep.world)
        dw13 = torch.empty_like(w13)
        C.gemm_grouped_k(dH, x_recv, sl.offs_local, dw13, EPI_BF16, 1.0, 256)
        arena.barrier()                                       # input gradients and weight gradients are ready
        dlogits, _ = C.router_bwd(logits, probs, idx, dwts, counts, renorm, aux_alpha * gs, z_beta * gs)
        dx_router = mm_nn(dlogits, router_w)
        dx = C.ep_combine_local(slot, sh.dxs.view(torch.bfloat16, T * k, D), None, dx_router)
        drouter = mm_tn(dlogits, x)
        return (dx, drouter, dw13, dw2, (dout if has_add else None), None, None, None, None, None, None, None, None)


# ----------------------------------------------------------------------------
# all_to_all transport (NCCL baseline on CUDA, gloo on CPU): autograd through torch ops
# ----------------------------------------------------------------------------
class _A2A(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, send, recv, group):
        ctx.send, ctx.recv, ctx.group = send, recv, group
        out = x.new_empty((sum(recv),) + tuple(x.shape[1:]))
        dist.all_to_all_single(out, x.contiguous(), recv, send, group=group)
        return out

    @staticmethod
    def backward(ctx, g):
        out = g.new_empty((sum(ctx.send),) + tuple(g.shape[1:]))
        dist.all_to_all_single(out, g.contiguous(), ctx.send, ctx.recv, group=ctx.group)
        return out, None, None, None


def _a2a_meta(t: torch.Tensor, send, recv, group) -> torch.Tensor:
    out = t.new_empty((sum(recv),) + tuple(t.shape[1:]))
    dist.all_to_all_single(out, t.contiguous(), recv, send, group=group)
    return out


def _ep_moe_a2a(x, router_w, w13, w2, add, ep, k, capacity, renorm, aux_alpha, z_beta):
    T, D = x.shape
    E = router_w.shape[0]
    El = w13.shape[0]
    N, me = ep.world, ep.rank
    logits = x.float() @ router_w.float().t()
    idx, w, probs = route_torch(logits, k, renorm)
    counts = torch.bincount(idx.reshape(-1), minlength=E).to(torch.int32)
    lay = ep_layout(ep.all_gather_counts(counts), me, El, capacity)
    lr = local_ranks(idx, E)
    flat_e = idx.reshape(-1)
    keep_lim = torch.as_tensor(lay.keep_lim, device=x.device)
    dst_base = torch.as_tensor(lay.dst_base, device=x.device)
    keep = lr.reshape(-1) < keep_lim[flat_e]
    pair = torch.nonzero(keep).squeeze(1)
    e_k = flat_e[pair]
    owner = e_k // El
    row = dst_base[e_k] + lr.reshape(-1)[pair]
    order = torch.argsort(owner * (1 << 40) + row)          # by owner, then destination row
    pair, owner, row = pair[order], owner[order], row[order]
    send = torch.bincount(owner, minlength=N).tolist()
    recv_counts = lay.kept[:, me * El:(me + 1) * El].sum(1)
    recv = [int(c) for c in recv_counts]
    xs = x.index_select(0, pair // k)
    xr = _A2A.apply(xs, send, recv, ep.group)
    rr = _a2a_meta(row, send, recv, ep.group).long()
    R = lay.rows[me]
    x_recv = x.new_zeros(R, D).index_copy(0, rr, xr)
    # one grouped GEMM per projection over the local experts' (128-padded) segments
    offs = torch.as_tensor(lay.offs_local[1:], dtype=torch.int32, device=x.device)
    h = torch._grouped_mm(x_recv, w13.transpose(-2, -1), offs=offs)
    g, u = deinterleave_cols(h)
    y_recv = torch._grouped_mm(F.silu(g) * u, w2.transpose(-2, -1), offs=offs)
    yb = _A2A.apply(y_recv.index_select(0, rr), recv, send, ep.group)
    # weighted sum of each token's k expert rows (dropped pairs contribute zero rows)
    yk = x.new_zeros(T * k, D).index_copy(0, pair, yb)
    out = torch.bmm(w.to(x.dtype).unsqueeze(1), yk.view(T, k, D)).squeeze(1)
    if add is not None:
        out = out + add
    aux = x.new_zeros((), dtype=torch.float32)
    if aux_alpha > 0:
        f = (counts.float() / (T * k)).detach()
        aux = aux + aux_alpha * E * (f * probs.mean(0)).sum()
    if z_beta > 0:
        lse = torch.logsumexp(logits, dim=-1)
        aux = aux + z_beta * (lse * lse).mean()
    return out, aux


def ep_moe_ffn(x: torch.Tensor, router_w: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, k: int, ep: EPContext,
               capacity: int = 0, renorm: bool = True, aux_alpha: float = 0.0, z_beta: float = 0.0,
               add: torch.Tensor | None = None, aux_grad_scale: float = 1.0):
    """Expert-parallel routed SwiGLU FFN.  x [T, D] local tokens; router_w [E, D]
    (replicated); w13 [El, 2F, D] / w2 [El, D, F] this rank's experts.  `capacity`
    is the per-expert limit over the whole group (0: dropless)."""
    if ep.transport == "p2p" and x.is_cuda and ep.layout == "device":
        # training (this layer's backward will read its forward slabs) or inference (slabs shared)
        train = torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (x, router_w, w13, w2))
        return _EPMoEDev.apply(x, router_w, w13, w2, add, ep, k, capacity, renorm, aux_alpha, z_beta,
                               aux_grad_scale, train)
    if ep.transport == "p2p" and x.is_cuda:
        return _EPMoEP2P.apply(x, router_w, w13, w2, add, ep, k, capacity, renorm, aux_alpha, z_beta,
                               aux_grad_scale)
    return _ep_moe_a2a(x, router_w, w13, w2, add, ep, k, capacity, renorm, aux_alpha, z_beta)
