"""Tensor helpers (reference src/omnicoder/utils/torchutils.py:102-678).

The reference's "safe_*" helpers exist to keep its torch.compile / CUDA-graph
traces stable; here they are plain, well-defined utilities:
  safe_new_like / safe_copy_into / safe_concat / safe_make_contiguous
  guard_shape(t, shape)            raises with a readable message (None = any size)
  safe_torch_save(obj, path)       atomic save (temp file + rename), retrying with the
                                   legacy (non-zip) serializer if the first attempt fails
  cuda_graph_capture_report(fn)    captures fn in a CUDA graph and reports success,
                                   node count and the error text of a failed capture
"""
from __future__ import annotations

import os
import tempfile

import torch


def safe_new_like(t: torch.Tensor, shape=None, dtype=None, fill: float | None = None) -> torch.Tensor:
    out = torch.empty(shape if shape is not None else t.shape, dtype=dtype or t.dtype, device=t.device)
    if fill is not None:
        out.fill_(fill)
    return out


def safe_copy_into(dst: torch.Tensor, src: torch.Tensor) -> torch.Tensor:
    if dst.shape != src.shape:
        raise ValueError(f"copy shape mismatch: {tuple(dst.shape)} <- {tuple(src.shape)}")
    return dst.copy_(src.to(dst.dtype))


def safe_concat(tensors, dim: int = 0) -> torch.Tensor:
    ts = [t for t in tensors if t is not None and t.numel() > 0]
    if not ts:
        raise ValueError("nothing to concatenate")
    dt = torch.result_type(*ts) if len(ts) > 1 else ts[0].dtype
    return torch.cat([t.to(dt) for t in ts], dim)


def safe_make_contiguous(t: torch.Tensor) -> torch.Tensor:
    return t if t.is_contiguous() else t.contiguous()


def guard_shape(t: torch.Tensor, shape, name: str = "tensor") -> torch.Tensor:
    if t.dim() != len(shape) or any(s is not None and s != d for s, d in zip(shape, t.shape)):
        raise ValueError(f"{name}: expected shape {tuple(shape)}, got {tuple(t.shape)}")
    return t


def safe_torch_save(obj, path: str) -> None:
    d = os.path.dirname(os.path.abspath(path))
    os.makedirs(d, exist_ok=True)
    fd, tmp = tempfile.mkstemp(dir=d, suffix=".tmp")
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


def cuda_graph_capture_report(fn, warmup: int = 2) -> dict:
    if not torch.cuda.is_available():
        return {"captured": False, "error": "CUDA not available"}
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    try:
        with torch.cuda.stream(s):
            for _ in range(warmup):
                fn()
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            fn()
        return {"captured": True, "graph": g}
    except Exception as e:  # report, do not raise
        return {"captured": False, "error": repr(e)}
