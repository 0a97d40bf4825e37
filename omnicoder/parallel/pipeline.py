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
Sends are non-blocking (isend), receives blocking, and every rank issues its
point-to-point operations in schedule order, so neighbouring stages never wait
on each other's sends.  The last stage owns the loss (mean over micro-batches);
`step()` returns it on every stage (broadcast from the last).

Optimiser: FusedAdamW over the stage's parameters with the global-norm clip
computed over all stages (one all-reduce of the squared norm).

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

    def forward(self, x, seq: int):
        """Stage 0: token ids [b, S] -> hidden; other stages: hidden [b*S, D] -> hidden;
        last stage returns final normalised hidden states."""
        if self.first:
            b, S = x.shape
            if x.is_cuda:
                self.rope.to(x.device)
            h = embedding(x.reshape(-1), self.embed)
        else:
            h = x
            if h.is_cuda:
                self.rope.to(h.device)
        positions = torch.arange(seq, device=h.device).repeat(h.shape[0] // seq)
        for blk in self.blocks:
            h, _ = blk(h, self.rope, positions, seq)
        return self.norm_f(h) if self.last else h


class PipelineTrainer:
    def __init__(self, model: OmniLM, tcfg, group=None, n_micro: int = 4):
        self.group = group if group is not None else dist.group.WORLD
        self.stage_id = dist.get_rank(self.group)
        self.P = dist.get_world_size(self.group)
        self.stage = PipelineStage(model, self.stage_id, self.P)
        self.tcfg, self.n_micro = tcfg, n_micro
        self.opt = FusedAdamW(self.stage.parameters(), lr=tcfg.lr, betas=tuple(tcfg.betas), eps=tcfg.eps,
                              weight_decay=tcfg.weight_decay, max_grad_norm=0.0)
        self.step_idx = 0
        self._peer = lambda s: dist.get_global_rank(self.group, s) if self.group is not dist.group.WORLD else s

    # ---- point-to-point -----------------------------------------------------
    def _send(self, t: torch.Tensor, to_stage: int, pending: list):
        pending.append(dist.isend(t.contiguous(), self._peer(to_stage), group=self.group))

    def _recv(self, shape, dtype, device, from_stage: int) -> torch.Tensor:
        t = torch.empty(shape, dtype=dtype, device=device)
        dist.recv(t, self._peer(from_stage), group=self.group)
        return t

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
        pending: list = []
        loss_sum = torch.zeros((), device=dev, dtype=torch.float32)

        def fwd(i):
            nonlocal loss_sum
            if st.first:
                x = ids_m[i]
            else:
                x = self._recv((mb * S, D), dtype, dev, self.stage_id - 1).requires_grad_(True)
            out = st(x, S)
            if st.last:
                loss = lm_head_cross_entropy(out, st.lm_head, lab_m[i].reshape(-1)) / M
                loss_sum = loss_sum + loss.detach().float()
                saved[i] = (x, loss)
            else:
                self._send(out.detach(), self.stage_id + 1, pending)
                saved[i] = (x, out)

        def bwd(i):
            x, out = saved.pop(i)
            if st.last:
                out.backward()
            else:
                g = self._recv(out.shape, out.dtype, dev, self.stage_id + 1)
                out.backward(g)
            if not st.first:
                self._send(x.grad, self.stage_id - 1, pending)

        warm = min(P - self.stage_id - 1, M)
        for i in range(warm):
            fwd(i)
        for i in range(M - warm):
            fwd(i + warm)
            bwd(i)
        for i in range(M - warm, M):
            bwd(i)
        for r in pending:
            r.wait()
        # global-norm clip over all stages, then the optimiser step
        scale = 1.0
        if self.tcfg.grad_clip > 0:
            sq = torch.zeros((), device=dev)
            for p in st.parameters():
                if p.grad is not None:
                    sq += p.grad.float().pow(2).sum()
            dist.all_reduce(sq, group=self.group)
            scale = min(1.0, self.tcfg.grad_clip / (float(sq.sqrt()) + 1e-6))
        lr = cosine_lr(self.step_idx, self.tcfg.lr, self.tcfg.warmup_steps, self.tcfg.max_steps)
        self.opt.step(lr=lr, grad_scale=scale)
        self.opt.zero_grad()
        self.step_idx += 1
        dist.broadcast(loss_sum, self._peer(P - 1), group=self.group)
        return loss_sum
