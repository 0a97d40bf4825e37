"""Loader of the in-tree sm_100a extension ``omnicoder._C``.

On a machine with a CUDA device the extension is mandatory: a missing or stale
build raises instead of silently falling back to PyTorch.  On CPU-only machines
the ops in :mod:`omnicoder.ops` run their PyTorch reference implementations,
which are also the fp32 oracles of the kernel tests.
"""
from __future__ import annotations

import importlib

import torch

_C = None
_ERR: Exception | None = None


def load():
    """Return the extension module, importing it on first use."""
    global _C, _ERR
    if _C is not None:
        return _C
    try:
        _C = importlib.import_module("omnicoder._C")
    except Exception as e:  # pragma: no cover - depends on the build
        _ERR = e
        raise RuntimeError(
            "omnicoder: the sm_100a extension omnicoder._C is not built or failed to load "
            "(run `python setup.py build_ext --inplace`): " + repr(e)
        ) from e
    return _C


def available() -> bool:
    try:
        load()
        return True
    except RuntimeError:
        return False


def use_cuda(t: torch.Tensor) -> bool:
    """True when `t` lives on a CUDA device; then the extension must be used."""
    if t.is_cuda:
        load()
        return True
    return False


def check_status():
    """Raise if any kernel recorded an error (timed-out wait, bad index)."""
    C = load()
    code, info, count = C.status()
    if code != 0:
        C.status_reset()
        names = {1: "timeout waiting for a free pipeline stage", 2: "timeout waiting for TMA data",
                 3: "timeout waiting for the epilogue", 4: "timeout waiting for the MMA",
                 5: "timeout waiting for a peer GPU flag", 6: "index out of bounds (access skipped)",
                 7: "timeout draining tensor-core work", 8: "timeout"}
        raise RuntimeError(f"omnicoder kernel error: {names.get(code, code)} (info={info}, count={count})")
