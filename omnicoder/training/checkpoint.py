"""Checkpoint save / load / resume.

* `save_checkpoint` writes atomically (temporary file + rename) with a
  `.meta.json` sidecar, like the reference's `save_with_sidecar` and
  `safe_torch_save` (src/omnicoder/utils/checkpoint.py:12-97,
  src/omnicoder/utils/torchutils.py:302-345).
* `maybe_load_checkpoint` accepts the dictionary shapes the reference loader
  accepts (`state_dict` / `model` / `module` nesting, `module.` / `_orig_mod.` /
  `model.` prefixes; src/omnicoder/inference/generate.py:3279-3370), loads
  non-strict, reports coverage, and understands this framework's exported
  layout (separate SwiGLU w1/w3) as well as its native one.
* Sharded optimiser state (ZeRO-1): one file per rank plus an index JSON,
  see `save_sharded_optimizer` / `load_sharded_optimizer`.
* `load_best_or_latest` / `maybe_save_best` keep a `_best.pt` by metric
  (src/omnicoder/utils/checkpoint.py:128-190).
"""
from __future__ import annotations

import glob
import json
import os
import tempfile
import time
from typing import Any

import torch

PREFIXES = ("module.", "_orig_mod.", "model.")


def _atomic_save(obj: Any, path: str):
    d = os.path.dirname(os.path.abspath(path)) or "."
    os.makedirs(d, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=d, prefix=".tmp_", suffix=".pt")
    os.close(fd)
    try:
        try:
            torch.save(obj, tmp)
        except Exception:
            torch.save(obj, tmp, _use_new_zipfile_serialization=False)
        os.replace(tmp, path)
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)


def save_checkpoint(path: str, model: torch.nn.Module, trainer_state: dict | None = None, meta: dict | None = None,
                    export: bool = False):
    sd = model.export_state_dict() if (export and hasattr(model, "export_state_dict")) else model.state_dict()
    obj = {"model": {k: v.detach().cpu() for k, v in sd.items()}}
    if trainer_state is not None:
        obj["trainer"] = trainer_state
    if hasattr(model, "cfg"):
        obj["config"] = model.cfg.to_dict()
    _atomic_save(obj, path)
    side = {"saved_at": time.time(), "format": "export" if export else "native", **(meta or {})}
    if hasattr(model, "cfg"):
        side["config"] = model.cfg.to_dict()
    with open(path + ".meta.json", "w") as f:
        json.dump(side, f, indent=1, default=str)
    return path


def _pick_state_dict(obj: Any) -> dict:
    if isinstance(obj, dict):
        for key in ("model", "state_dict", "module", "model_state_dict", "weights"):
            if key in obj and isinstance(obj[key], dict):
                return _pick_state_dict(obj[key])
        if all(isinstance(v, torch.Tensor) for v in obj.values()):
            return obj
    raise ValueError("no state_dict found in checkpoint")


def normalize_keys(sd: dict) -> dict:
    out = {}
    for k, v in sd.items():
        kk = k
        changed = True
        while changed:
            changed = False
            for p in PREFIXES:
                if kk.startswith(p):
                    kk = kk[len(p):]
                    changed = True
            kk = kk.replace("._orig_mod.", ".")
        out[kk] = v
    return out


def maybe_load_checkpoint(model: torch.nn.Module, ckpt_path: str | None, strict: bool = False) -> dict:
    """Load weights into `model`; returns a coverage report."""
    if not ckpt_path:
        return {"loaded": False}
    obj = torch.load(ckpt_path, map_location="cpu", weights_only=False)
    sd = normalize_keys(_pick_state_dict(obj))
    if any(k.endswith(".w1") for k in sd) and hasattr(model, "load_export_state_dict"):
        res = model.load_export_state_dict(sd, strict=strict)
    else:
        own = model.state_dict()
        sd = {k: v.to(own[k].dtype) for k, v in sd.items() if k in own and own[k].shape == v.shape}
        res = model.load_state_dict(sd, strict=strict)
    missing = list(getattr(res, "missing_keys", []))
    unexpected = list(getattr(res, "unexpected_keys", []))
    total = len(model.state_dict())
    return {"loaded": True, "missing": missing, "unexpected": unexpected,
            "coverage": 1.0 - len(missing) / max(1, total)}


# ---- sharded optimiser state (ZeRO-1) ------------------------------------------
def save_sharded_optimizer(dirpath: str, rank: int, world: int, state: dict, step: int):
    os.makedirs(dirpath, exist_ok=True)
    _atomic_save(state, os.path.join(dirpath, f"optim_rank{rank:05d}_of_{world:05d}.pt"))
    if rank == 0:
        with open(os.path.join(dirpath, "optim_index.json"), "w") as f:
            json.dump({"world": world, "step": step,
                       "files": [f"optim_rank{r:05d}_of_{world:05d}.pt" for r in range(world)]}, f, indent=1)


def load_sharded_optimizer(dirpath: str, rank: int, world: int) -> dict:
    with open(os.path.join(dirpath, "optim_index.json")) as f:
        idx = json.load(f)
    if idx["world"] != world:
        raise ValueError(f"optimizer state was saved with world={idx['world']}, now world={world}")
    return torch.load(os.path.join(dirpath, idx["files"][rank]), map_location="cpu", weights_only=False)


# ---- best / latest ---------------------------------------------------------------
def maybe_save_best(path: str, model: torch.nn.Module, metric: float, higher_is_better: bool = False) -> bool:
    best = os.path.splitext(path)[0] + "_best.pt"
    side = best + ".meta.json"
    prev = None
    if os.path.exists(side):
        try:
            prev = json.load(open(side)).get("metric")
        except Exception:
            prev = None
    better = prev is None or (metric > prev if higher_is_better else metric < prev)
    if better:
        save_checkpoint(best, model, meta={"metric": metric})
    return better


def load_best_or_latest(model: torch.nn.Module, directory_or_path: str) -> str | None:
    p = directory_or_path
    if os.path.isdir(p):
        best = sorted(glob.glob(os.path.join(p, "*_best.pt")))
        cands = best or sorted(glob.glob(os.path.join(p, "*.pt")), key=os.path.getmtime)
        if not cands:
            return None
        p = cands[-1]
    if not os.path.exists(p):
        return None
    maybe_load_checkpoint(model, p)
    return p


# ----------------------------------------------------------------------------
# sidecars, manifest, best-weights registry (reference src/omnicoder/utils/
# checkpoint.py:12-224 save_with_sidecar, model_manifest.py, best_weights.py)
# ----------------------------------------------------------------------------
def save_with_sidecar(path: str, model: torch.nn.Module, meta: dict | None = None, vocab=None) -> None:
    """state_dict (CPU copy, atomic) + `<path>.meta.json` (config, parameter count, user meta)
    + optional `<path>.vocab.json` (the unified-vocabulary sidecar)."""
    import json
    sd = {k: v.detach().cpu() for k, v in model.state_dict().items()}
    _atomic_save({"model": sd, "config": getattr(model, "cfg").to_dict() if hasattr(model, "cfg") else None}, path)
    info = {"params": int(sum(v.numel() for v in sd.values())), "keys": len(sd)}
    if hasattr(model, "cfg"):
        info["config"] = model.cfg.to_dict()
    info.update(meta or {})
    with open(path + ".meta.json", "w") as f:
        json.dump(info, f, indent=1)
    if vocab is not None:
        vocab.save(path + ".vocab.json")


def write_manifest(directory: str) -> dict:
    """manifest.json of every checkpoint file in `directory` (bytes, mtime, meta if present)."""
    import json
    out = {}
    for f in sorted(os.listdir(directory)):
        p = os.path.join(directory, f)
        if f.endswith((".pt", ".pth")) and os.path.isfile(p):
            e = {"bytes": os.path.getsize(p), "mtime": os.path.getmtime(p)}
            if os.path.exists(p + ".meta.json"):
                e["meta"] = json.load(open(p + ".meta.json"))
            out[f] = e
    with open(os.path.join(directory, "manifest.json"), "w") as fh:
        json.dump(out, fh, indent=1)
    return out


class BestWeightsRegistry:
    """Tracks the best checkpoint per task in a JSON file: register(task, path, metric)."""

    def __init__(self, path: str, higher_is_better: bool = True):
        import json
        self.path, self.hib = path, higher_is_better
        self.data = json.load(open(path)) if os.path.exists(path) else {}

    def register(self, task: str, ckpt: str, metric: float) -> bool:
        import json
        cur = self.data.get(task)
        better = cur is None or (metric > cur["metric"] if self.hib else metric < cur["metric"])
        if better:
            self.data[task] = {"path": ckpt, "metric": float(metric)}
            tmp = self.path + ".tmp"
            with open(tmp, "w") as f:
                json.dump(self.data, f, indent=1)
            os.replace(tmp, self.path)
        return better

    def best(self, task: str) -> str | None:
        e = self.data.get(task)
        return e["path"] if e else None
