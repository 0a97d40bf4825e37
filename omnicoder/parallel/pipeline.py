"""Pipeline parallelism: contiguous layer stages, 1F1B schedule, activations and
their gradients exchanged with torch.distributed point-to-point operations (NCCL
on GPUs, gloo on CPU).

Stage s of P holds blocks [s L / P, (s + 1) L / P); stage 0 also the embedding,
the last stage the final norm and the LM head.  A step splits the batch into M
micro-batches and runs the one-forward-one-backward schedule:
  warm-up:  min(P - s - 1, M) forwards
  steady:   forward of micro-batch i + warm-up, backward of micro-batch i
  cool-down: remaining backwards
which bounds the activations a stage keeps alive to P - s micro-batches.
Every exchange is one batched point-to-point call (`batch_isend_irecv`): a send
alone, a receive alone, or the send of this micro-batch's output paired with the
receive of the next gradient (and the send of a gradient paired with the receive of
the next input) -- the pairing of 1F1B schedules.  NCCL serialises unbatched
point-to-point operations of a communicator, and separately issued send / receive
pairs of neighbouring stages then wait on each other; batched pairs do not.  The last stage owns the loss (mean over micro-batches);
`step()` returns it on every stage (broadcast from the last).

Optimiser: FusedAdamW over the stage's parameters with the global-norm clip
computed over all stages (one all-reduce of the squared norm).

Tensor parallelism inside the stages (`tp`, an omnicoder.parallel.tensor.TensorParallel
over the stage's ranks, the model built with it): a stage is a TP group, the
activations crossing stages are the sequence-parallel token shards (rank t of a
stage exchanges with rank t of the next), replicated gradients are summed over
the TP group and the clip norm counts each replicated parameter once per stage.

The reference has no pipeline parallelism.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..models.lm import OmniLM
from ..ops import FusedAdamW, cosine_lr, embedding, lm_head_cross_entropy


class PipelineStage(torch.nn.Module):
    def __init__(self, model: OmniLM, stage: int, n_stages: int):
        super().__init__()
        L = len(model.blocks)
        if L % n_stages:
            raise ValueError(f"{L} layers do not split into {n_stages} pipeline stages")
        if model.cfg.tie_embeddings and n_stages > 1:
            raise ValueError("pipeline parallelism needs untied embeddings (embedding and head live on different stages)")
        per = L // n_stages
        self.stage, self.n_stages, self.cfg = stage, n_stages, model.cfg
        self.first, self.last = stage == 0, stage == n_stages - 1
        self.blocks = torch.nn.ModuleList(list(model.blocks)[stage * per:(stage + 1) * per])
        self.embed = model.embed if self.first else None
        self.norm_f = model.norm_f if self.last else None
        self.lm_head = model.lm_head if self.last else None
        self.rope = model.rope
        self.tp = model.tp                      # TPContext of the stage's tensor-parallel group, or None

    def forward(self, x, seq: int, batch: int | None = None):
        """Stage 0: token ids [b, S] -> hidden; other stages: hidden [b*S (/ TP), D] -> hidden;
        last stage returns final normalised hidden states (this rank's token shard with TP)."""
        if self.first:
            b, S = x.shape
            batch = b
            if x.is_cuda:
                self.rope.to(x.device)
            flat = x.reshape(-1)
            if self.tp is not None:
                from .tensor import scatter_seq
                flat = scatter_seq(flat, self.tp)
            h = embedding(flat, self.embed)
        else:
            h = x
            if h.is_cuda:
                self.rope.to(h.device)
        if batch is None:
            batch = h.shape[0] // seq
        positions = torch.arange(seq, device=h.device).repeat(batch)
        for blk in self.blocks:
            h, _ = blk(h, self.rope, positions, seq)
        return self.norm_f(h) if self.last else h


class PipelineTrainer:
    def __init__(self, model: OmniLM, tcfg, group=None, n_micro: int = 4, tp=None):
        """`group`: the ranks of this rank's pipeline (one per stage); `tp`: the TensorParallel
        layout of this rank's stage (the model must have been built with it)."""
        self.group = group if group is not None else dist.group.WORLD
        self.stage_id = dist.get_rank(self.group)
        self.P = dist.get_world_size(self.group)
        self.tp = tp
        self.tp_world = tp.world if tp is not None else 1
        self.stage = PipelineStage(model, self.stage_id, self.P)
        if tp is not None:
            self.replicated = [p for p in self.stage.parameters() if not getattr(p, "tp_sharded", False)]
            self.sharded = [p for p in self.stage.parameters() if getattr(p, "tp_sharded", False)]
        self.tcfg, self.n_micro = tcfg, n_micro
        self.opt = FusedAdamW(self.stage.parameters(), lr=tcfg.lr, betas=tuple(tcfg.betas), eps=tcfg.eps,
                              weight_decay=tcfg.weight_decay, max_grad_norm=0.0)
        self.step_idx = 0
        self._peer = lambda s: dist.get_global_rank(self.group, s) if self.group is not dist.group.WORLD else s

    # ---- point-to-point -----------------------------------------------------
    def _p2p(self, send: torch.Tensor | None = None, send_to: int = -1, recv_like: tuple | None = None,
             recv_from: int = -1) -> torch.Tensor | None:
        """One batched exchange: optionally send `send` to stage send_to and receive a tensor of
        recv_like = (shape, dtype, device) from stage recv_from."""
        ops, out = [], None
        if send is not None:
            ops.append(dist.P2POp(dist.isend, send.contiguous(), self._peer(send_to), group=self.group))
        if recv_like is not None:
            out = torch.empty(recv_like[0], dtype=recv_like[1], device=recv_like[2])
            ops.append(dist.P2POp(dist.irecv, out, self._peer(recv_from), group=self.group))
        if ops:
            for r in dist.batch_isend_irecv(ops):
                r.wait()
        return out

    # ---- one optimiser step ------------------------------------------------
    def step(self, ids: torch.Tensor, labels: torch.Tensor):
        st, P, M = self.stage, self.P, self.n_micro
        B, S = ids.shape
        if B % M:
            raise ValueError(f"batch {B} does not split into {M} micro-batches")
        mb = B // M
        dev = ids.device
        D = self.stage.cfg.d_model
        dtype = next(self.stage.parameters()).dtype
        ids_m, lab_m = ids.chunk(M), labels.chunk(M)
        saved: dict[int, tuple] = {}
        loss_sum = torch.zeros((), device=dev, dtype=torch.float32)

        rows = mb * S // self.tp_world
        first, last = st.first, st.last
        prev, nxt = self.stage_id - 1, self.stage_id + 1
        act_like = ((rows, D), dtype, dev)

        def forward(i, x):
            nonlocal loss_sum
            if first:
                x = ids_m[i]
            else:
                x = x.requires_grad_(True)
            out = st(x, S, mb)
            if last:
                lab = lab_m[i].reshape(-1)
                if self.tp is not None:
                    from .tensor import scatter_seq
                    lab = scatter_seq(lab, self.tp.tp)
                loss = lm_head_cross_entropy(out, st.lm_head, lab) / M
                loss_sum = loss_sum + loss.detach().float()
                saved[i] = (x, loss)
                return None
            saved[i] = (x, out)
            return out.detach()

        def backward(i, g):
            x, out = saved.pop(i)
            if last:
                out.backward()
            else:
                out.backward(g)
            return None if first else x.grad

        recv_fwd = lambda: None if first else self._p2p(recv_like=act_like, recv_from=prev)
        warm = min(P - self.stage_id - 1, M)
        for i in range(warm):                                   # warm-up forwards
            out = forward(i, recv_fwd())
            self._p2p(send=out, send_to=nxt)
        rem = M - warm
        x = recv_fwd() if rem > 0 else None
        for j in range(rem):                                    # steady state: one forward, one backward
            out = forward(warm + j, x)
            g = None if last else self._p2p(send=out, send_to=nxt, recv_like=act_like, recv_from=nxt)
            dx = backward(j, g)
            if j == rem - 1:
                if not first:
                    self._p2p(send=dx, send_to=prev)
            elif first:
                x = None
            else:
                x = self._p2p(send=dx, send_to=prev, recv_like=act_like, recv_from=prev)
        for j in range(rem, M):                                 # cool-down backwards
            g = None if last else self._p2p(recv_like=act_like, recv_from=nxt)
            dx = backward(j, g)
            if not first:
                self._p2p(send=dx, send_to=prev)
        # global-norm clip over all stages, then the optimiser step
        scale = 1.0
        if self.tp is not None:
            # each TP rank back-propagated the mean loss of its own token shard: sum the replicated
            # gradients over the stage's group and average everything over it
            self.tp.replicated, self.tp.sharded = self.replicated, self.sharded
            self.tp.sync_grads()
            scale = 1.0 / self.tp_world
        if self.tcfg.grad_clip > 0:
            sq = torch.zeros((), device=dev)
            if self.tp is None:
                for p in st.parameters():
                    if p.grad is not None:
                        sq += p.grad.float().pow(2).sum()
            else:
                for p in self.sharded:
                    if p.grad is not None:
                        sq += p.grad.float().pow(2).sum()
                dist.all_reduce(sq, group=self.tp.group)
                for p in self.replicated:
                    if p.grad is not None:
                        sq += p.grad.float().pow(2).sum()
            dist.all_reduce(sq, group=self.group)
            norm = float(sq.sqrt()) * scale
            scale *= min(1.0, self.tcfg.grad_clip / (norm + 1e-6))
        lr = cosine_lr(self.step_idx, self.tcfg.lr, self.tcfg.warmup_steps, self.tcfg.max_steps)
        self.opt.step(lr=lr, grad_scale=scale)
        self.opt.zero_grad()
        self.step_idx += 1
        if self.tp is not None and st.last:
            dist.all_reduce(loss_sum, group=self.tp.group)
            loss_sum = loss_sum / self.tp_world
        dist.broadcast(loss_sum, self._peer(P - 1), group=self.group)
        return loss_sum
