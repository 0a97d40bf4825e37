"""Restart from the last good checkpoint.

CheckpointManager keeps `keep` step checkpoints (model weights + trainer state:
step, optimiser moments) in one directory, each written to a temporary file
and renamed into place, so a crash mid-save never leaves a half-written file
under a checkpoint's name (`save_async` copies the state to host memory and writes
on a background thread).  `load_latest` tries the newest first and falls
back to older ones when a file is unreadable (truncated, corrupted), logging
each rejected file.

`train_with_recovery` is the loop a relaunched job runs: resume from the
latest good checkpoint, then for each step run the fault injector's hook,
check the group's health (when a Heartbeat is given: every rank announces the
step and waits for the others' announcements), train and save every
`save_every` steps.  Relaunch itself is the launcher's job
(`torch.distributed.run --max-restarts`, `omnicoder.tools.torchrun_ep
--max_restarts`).  The reference saves plain state_dicts and re-creates its
optimiser after loading the saved state (src/omnicoder/training/pretrain.py:497-516,582),
so a resumed run there restarts the moments from zero.
"""
from __future__ import annotations

import glob
import logging
import os
import re
import threading
from typing import Callable

import torch

from .checkpoint import _atomic_save

log = logging.getLogger("omnicoder.resilience")


class CheckpointManager:
    def __init__(self, directory: str, keep: int = 3, rank: int = 0):
        self.dir, self.keep, self.rank = directory, max(1, keep), rank
        os.makedirs(directory, exist_ok=True)

    def _path(self, step: int) -> str:
        return os.path.join(self.dir, f"step_{step:09d}.rank{self.rank}.pt")

    def steps(self) -> list[int]:
        pat = re.compile(rf"step_(\d+)\.rank{self.rank}\.pt$")
        found = [int(m.group(1)) for p in glob.glob(os.path.join(self.dir, f"step_*.rank{self.rank}.pt"))
                 if (m := pat.search(p))]
        return sorted(found)

    def _snapshot(self, step, model, trainer) -> dict:
        # copy=True: for CPU tensors .cpu() would alias the live weights
        return {"step": step, "model": {k: v.detach().to("cpu", copy=True) for k, v in model.state_dict().items()},
                "trainer": _to_cpu(trainer.state_dict())}

    def _write(self, step: int, obj: dict) -> str:
        path = self._path(step)
        _atomic_save(obj, path)
        for old in self.steps()[:-self.keep]:
            os.unlink(self._path(old))
        return path

    def save(self, step: int, model: torch.nn.Module, trainer) -> str:
        self.wait()
        return self._write(step, self._snapshot(step, model, trainer))

    def save_async(self, step: int, model: torch.nn.Module, trainer) -> None:
        """Copy the state to host memory now (training may continue and change the device
        tensors afterwards) and write the file on a background thread; at most one write is in
        flight (a new save first waits for the previous one)."""
        self.wait()
        obj = self._snapshot(step, model, trainer)
        self._error = None

        def run():
            try:
                self._write(step, obj)
            except Exception as e:          # surfaced by wait()
                self._error = e

        self._thread = threading.Thread(target=run, name="omnicoder-ckpt", daemon=False)
        self._thread.start()

    def wait(self) -> None:
        t = getattr(self, "_thread", None)
        if t is not None:
            t.join()
            self._thread = None
        err = getattr(self, "_error", None)
        if err is not None:
            self._error = None
            raise err

    def load_latest(self, model: torch.nn.Module, trainer) -> int:
        """Load the newest readable checkpoint; returns its step (0 when there is none)."""
        self.wait()
        for step in reversed(self.steps()):
            path = self._path(step)
            try:
                obj = torch.load(path, map_location="cpu", weights_only=False)
                model.load_state_dict(obj["model"])
                trainer.load_state_dict(_to_device(obj["trainer"], next(model.parameters()).device))
                return int(obj["step"])
            except Exception as e:                                    # unreadable: try the previous one
                log.warning("checkpoint %s rejected (%s); trying an older one", path, e)
        return 0


def _to_cpu(x):
    if isinstance(x, torch.Tensor):
        return x.detach().to("cpu", copy=True)
    if isinstance(x, dict):
        return {k: _to_cpu(v) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return type(x)(_to_cpu(v) for v in x)
    return x


def _to_device(x, device):
    if isinstance(x, torch.Tensor):
        return x.to(device)
    if isinstance(x, dict):
        return {k: _to_device(v, device) for k, v in x.items()}
    if isinstance(x, (list, tuple)):
        return type(x)(_to_device(v, device) for v in x)
    return x


def train_with_recovery(trainer, batch_fn: Callable[[int], tuple], steps: int, ckpt: CheckpointManager,
                        save_every: int = 100, heartbeat=None, injector=None, rank: int = 0) -> dict:
    """Run steps [resume, steps) of `trainer`; batch_fn(step) -> (ids, labels).  Returns
    {"resumed_from", "losses"}.  RankFailure / InjectedFault propagate to the caller
    (after `heartbeat.leave()` so the other ranks see it)."""
    start = ckpt.load_latest(trainer.model, trainer)
    losses = []
    try:
        for step in range(start, steps):
            if injector is not None:
                injector.at_step(rank, step, heartbeat)
            if heartbeat is not None:
                heartbeat.check(step)
            ids, labels = batch_fn(step)
            losses.append(float(trainer.step(ids, labels).loss))
            if (step + 1) % save_every == 0 or step + 1 == steps:
                ckpt.save(step + 1, trainer.model, trainer)
    except Exception as e:
        if heartbeat is not None:
            heartbeat.leave(f"{type(e).__name__}: {e}")
        raise
    return {"resumed_from": start, "losses": losses}
