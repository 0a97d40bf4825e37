"""Exports for on-device runtimes other than ONNX: ExecuTorch, Core ML and MLC.

Reference: src/omnicoder/export/executorch_export.py, coreml_decode_export.py,
mlc_compile.py (each traces the decode step and hands it to that runtime's converter).

All three converters take a `torch.export` program of the decode-step function
(omnicoder.export.onnx_export.DecodeStepWrapper: token ids, position and KV-cache
tensors in, logits and updated caches out).  `export_program` writes that program
(`.pt2`, `torch.export.save`) -- it needs nothing beyond torch -- and each target then
converts it when its package is installed:

  executorch  to_edge -> to_executorch -> `.pte`              (package `executorch`)
  coreml      coremltools.convert(program) -> `.mlpackage`    (package `coremltools`)
  mlc         a compile recipe (`mlc_config.json`: model config, cache shapes, quantisation)
              for `mlc_llm compile`, written always; compiled when `mlc_llm` is importable.
A target whose package is missing is reported as skipped with the reason, never faked.
"""
from __future__ import annotations

import json
import os

import torch


def export_program(model, path: str, batch: int = 1, max_len: int = 256, tokens: int = 1):
    """torch.export program of the decode step (or of a `tokens`-token prefill) -> saved to `path`."""
    from .onnx_export import example_inputs
    w, args = example_inputs(model, batch, max_len, tokens)
    prog = torch.export.export(w, args, strict=False)
    torch.export.save(prog, path)
    return prog


def _available(mod: str) -> bool:
    import importlib
    try:
        importlib.import_module(mod)
        return True
    except ImportError:
        return False


def export_executorch(prog, path: str) -> dict:
    if not _available("executorch"):
        return {"skipped": "package `executorch` is not installed"}
    from executorch.exir import to_edge
    with open(path, "wb") as f:
        f.write(to_edge(prog).to_executorch().buffer)
    return {"file": path, "bytes": os.path.getsize(path)}


def export_coreml(prog, path: str) -> dict:
    if not _available("coremltools"):
        return {"skipped": "package `coremltools` is not installed"}
    import coremltools as ct
    ct.convert(prog).save(path)
    return {"file": path}


def mlc_recipe(model, out_dir: str, quantization: str = "q4f16_1", max_len: int = 4096) -> dict:
    """The model description `mlc_llm compile` needs (architecture sizes, cache layout, quantisation)."""
    from .onnx_export import spec_cache_shapes
    cfg = model.cfg
    recipe = {"model_type": "omnicoder", "quantization": quantization, "context_window_size": max_len,
              "config": cfg.to_dict(), "kv_cache": [list(s) for s in spec_cache_shapes(cfg, 1, max_len)[:2]],
              "io": {"inputs": ["input_ids", "position", "k_lat_i", "v_lat_i"],
                     "outputs": ["logits", "nk_lat_i", "nv_lat_i"]}}
    os.makedirs(out_dir, exist_ok=True)
    p = os.path.join(out_dir, "mlc_config.json")
    with open(p, "w") as f:
        json.dump(recipe, f, indent=1, default=str)
    out = {"recipe": p}
    if not _available("mlc_llm"):
        out["compile"] = "skipped: package `mlc_llm` is not installed"
    return out


def export_all(model, out_dir: str, max_len: int = 256, targets=("executorch", "coreml", "mlc")) -> dict:
    os.makedirs(out_dir, exist_ok=True)
    res = {}
    prog_path = os.path.join(out_dir, "decode_step.pt2")
    prog = export_program(model.eval(), prog_path, max_len=max_len)
    res["program"] = {"file": prog_path, "bytes": os.path.getsize(prog_path)}
    if "executorch" in targets:
        res["executorch"] = export_executorch(prog, os.path.join(out_dir, "decode_step.pte"))
    if "coreml" in targets:
        res["coreml"] = export_coreml(prog, os.path.join(out_dir, "decode_step.mlpackage"))
    if "mlc" in targets:
        res["mlc"] = mlc_recipe(model, out_dir, max_len=max_len)
    with open(os.path.join(out_dir, "runtimes_manifest.json"), "w") as f:
        json.dump(res, f, indent=1, default=str)
    return res
