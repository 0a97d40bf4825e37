"""Training step engine: forward, backward, gradient synchronisation, optimiser.

`Trainer.step(ids, labels)` is the public per-step API used by the pretraining
entry point, the benchmark and the tests.  With a process group it runs the
expert-parallel x data-parallel layout of :mod:`omnicoder.parallel` (experts
sharded over the EP group, dense parameters replicated with ZeRO-1 sharded
AdamW state); without one it is the single-device trainer.

`cuda_graph=True` (grad_accum 1; one device, or an expert x data parallel layout whose
exchange runs on the device -- see ExpertDataParallel.graph_capturable): after `graph_warmup` eager
steps, forward + backward is captured once as a CUDA graph and replayed every
step (the batch is copied into static input buffers; the gradients are static
tensors the replay overwrites, so they are not reset between steps); the
optimiser runs eagerly after the replay, with the learning rate of the step.
A capture that fails leaves the trainer in eager mode (`graph_error` says why).

The reference trainer's step (src/omnicoder/training/pretrain.py:915-952:
scaled backward, optimizer.step, zero_grad) has no gradient synchronisation at
all; it runs in a single process.
"""
from __future__ import annotations

import time
from dataclasses import dataclass

import torch

from ..config import ModelConfig, TrainConfig
from ..models.lm import OmniLM
from ..ops import FusedAdamW, cosine_lr


@dataclass
class StepStats:
    loss: torch.Tensor       # device scalar (no host sync)
    ce: torch.Tensor
    aux: torch.Tensor
    tokens: int
    lr: float


class Trainer:
    def __init__(self, model: OmniLM, tcfg: TrainConfig, parallel=None, cuda_graph: bool = False,
                 graph_warmup: int = 2):
        self.model = model
        self.tcfg = tcfg
        self.parallel = parallel
        self.step_idx = 0
        self.cuda_graph = (cuda_graph and max(1, tcfg.grad_accum) == 1 and
                           (parallel is None or getattr(parallel, "graph_capturable", lambda: False)()))
        self.graph_warmup = graph_warmup
        self._graph = None
        self._graph_key = None
        self.graph_error: str | None = None
        if parallel is not None:
            self.opt = parallel.make_optimizer(model, tcfg)
        else:
            self.opt = FusedAdamW(model.parameters(), lr=tcfg.lr, betas=tuple(tcfg.betas), eps=tcfg.eps,
                                  weight_decay=tcfg.weight_decay, max_grad_norm=tcfg.grad_clip)
        model.set_aux_grad_scale(1.0 / max(1, tcfg.grad_accum))

    def lr_at(self, step: int) -> float:
        t = self.tcfg
        return cosine_lr(step, t.lr, t.warmup_steps, t.max_steps)

    def step(self, ids: torch.Tensor, labels: torch.Tensor, assume_all_valid: bool = False) -> StepStats:
        """One optimiser step over micro-batches `ids`/`labels` [B, S] (split into
        grad_accum chunks along the batch)."""
        if self.cuda_graph and ids.is_cuda:
            key = (tuple(ids.shape), tuple(labels.shape), bool(assume_all_valid))
            if self._graph is None and self.step_idx >= self.graph_warmup:
                self._capture(ids, labels, assume_all_valid, key)
            if self._graph is not None and key == self._graph_key:
                return self._graph_step(ids, labels)
            if self._graph is not None:              # eager step beside the graph: fresh gradients
                self.opt.zero_grad(set_to_none=True)
        accum = max(1, self.tcfg.grad_accum)
        chunks_ids = ids.chunk(accum, dim=0)
        chunks_lab = labels.chunk(accum, dim=0)
        loss_sum = ce_sum = aux_sum = None
        for mi, (ci, cl) in enumerate(zip(chunks_ids, chunks_lab)):
            if self.parallel is not None:
                self.parallel.before_forward(mi, len(chunks_ids))
            out = self.model(ci, labels=cl, assume_all_valid=assume_all_valid)
            loss = out["loss"] / accum
            loss.backward()
            l, c, a = out["loss"].detach(), out["ce"].detach(), out["aux"].detach()
            loss_sum = l if loss_sum is None else loss_sum + l
            ce_sum = c if ce_sum is None else ce_sum + c
            aux_sum = a if aux_sum is None else aux_sum + a
        lr = self.lr_at(self.step_idx)
        if self.parallel is not None:
            self.parallel.sync_and_step(self.model, self.opt, lr)
        else:
            self.opt.step(lr=lr)
        self.opt.zero_grad(set_to_none=True)
        self.step_idx += 1
        return StepStats(loss_sum / accum, ce_sum / accum, aux_sum / accum, ids.numel(), lr)

    # ------------------------------------------------------------------
    def _capture(self, ids, labels, assume_all_valid, key):
        self._static_ids, self._static_lab = ids.clone(), labels.clone()
        self.opt.zero_grad(set_to_none=True)
        dev = ids.device
        par = self.parallel
        if par is not None:
            # gradient reductions move out of the backward hooks into opt.step(); the graph
            # holds only this rank's kernels (device-side exchange and barriers), no NCCL call
            par.set_deferred_reduce(True)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        try:
            with torch.cuda.stream(side):        # lazy setup outside the capture; no optimiser step
                if par is not None:
                    par.before_forward(0, 1)
                out = self.model(self._static_ids, labels=self._static_lab, assume_all_valid=assume_all_valid)
                out["loss"].backward()
            torch.cuda.current_stream(dev).wait_stream(side)
            del out
            self.opt.zero_grad(set_to_none=True)
            torch.cuda.synchronize(dev)
            torch.cuda.empty_cache()             # the graph's private pool replaces the eager steps' cache
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                if par is not None:
                    par.before_forward(0, 1)
                out = self.model(self._static_ids, labels=self._static_lab, assume_all_valid=assume_all_valid)
                out["loss"].backward()
        except Exception as e:                   # stay eager
            self.cuda_graph, self.graph_error = False, f"{type(e).__name__}: {e}"
            if par is not None:
                par.set_deferred_reduce(False)
            self.opt.zero_grad(set_to_none=True)
            return
        self._graph, self._graph_key = g, key
        self._static_out = (out["loss"].detach(), out["ce"].detach(), out["aux"].detach())
        self._static_grads = [(p, p.grad) for p in self.model.parameters() if p.grad is not None]

    def _graph_step(self, ids, labels) -> StepStats:
        self._static_ids.copy_(ids, non_blocking=True)
        self._static_lab.copy_(labels, non_blocking=True)
        self._graph.replay()
        for p, g in self._static_grads:              # the replay wrote these tensors
            p.grad = g
        lr = self.lr_at(self.step_idx)
        if self.parallel is not None:
            self.parallel.sync_and_step(self.model, self.opt, lr)
        else:
            self.opt.step(lr=lr)
        self.step_idx += 1
        loss, ce, aux = (t.clone() for t in self._static_out)
        return StepStats(loss, ce, aux, ids.numel(), lr)

    # ------------------------------------------------------------------
    def state_dict(self) -> dict:
        return {"step": self.step_idx, "optimizer": self.opt.state_dict()}

    def load_state_dict(self, sd: dict):
        self.step_idx = int(sd["step"])
        self.opt.load_state_dict(sd["optimizer"])


def synthetic_batch(batch: int, seq: int, vocab: int, seed: int, step: int, device="cpu", pin: bool = False):
    """Uniform random token ids (labels = ids shifted left by one, last label from the
    same stream).  Deterministic in (seed, step)."""
    g = torch.Generator(device="cpu")
    g.manual_seed(seed * 1_000_003 + step)
    stream = torch.randint(0, vocab, (batch, seq + 1), generator=g)
    ids, labels = stream[:, :-1].contiguous(), stream[:, 1:].contiguous()
    if pin:
        ids, labels = ids.pin_memory(), labels.pin_memory()
    if str(device) != "cpu":
        ids, labels = ids.to(device, non_blocking=True), labels.to(device, non_blocking=True)
    return ids, labels
