"""Mobile / edge package (reference src/omnicoder/export/mobile_packager.py:1-673).

package_model(model, out_dir): writes
  weights_int4.pt   every 2-D linear weight (except the embedding / head) in the
                    int4 format of omnicoder.quant.int4 (packed nibbles + per-row
                    scales), other tensors in fp16
  config.json       the model config
  vocab.json        the unified-vocabulary sidecar (text / image / video / audio ranges)
  decode_step.onnx  the ONNX decode step (only when the onnx package is importable)
  manifest.json     file list with sizes and sha256, format version, quantisation
load_package(out_dir, device) rebuilds a float model from the package.
Core ML / ExecuTorch / MLC targets need toolchains that are not installed here;
`export_targets()` reports which are available.
"""
from __future__ import annotations

import hashlib
import json
import os

import torch

FORMAT_VERSION = 1


def export_targets() -> dict:
    import importlib
    out = {}
    for name, mod in [("onnx", "onnx"), ("coreml", "coremltools"), ("executorch", "executorch"), ("mlc", "tvm")]:
        try:
            importlib.import_module(mod)
            out[name] = True
        except ImportError:
            out[name] = False
    return out


def _sha(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 20), b""):
            h.update(b)
    return h.hexdigest()


def package_model(model, out_dir: str, skip: tuple = ("embed", "head")) -> dict:
    from ..multimodal.vocab import VocabSidecar
    from ..quant.int4 import pack_int4
    os.makedirs(out_dir, exist_ok=True)
    packed = {}
    for name, t in model.state_dict().items():
        t = t.detach().float().cpu()
        if t.dim() == 2 and not any(s in name for s in skip):
            q, scale, _ = pack_int4(t)
            packed[name] = {"int4": q, "scale": scale.float(), "shape": list(t.shape)}
        else:
            packed[name] = {"fp16": t.half()}
    torch.save(packed, os.path.join(out_dir, "weights_int4.pt"))
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(model.cfg.to_dict(), f, indent=1)
    VocabSidecar.from_config(text_vocab=model.cfg.vocab_size).save(os.path.join(out_dir, "vocab.json"))
    if export_targets()["onnx"]:
        from .onnx_export import export_decode_step
        export_decode_step(model, os.path.join(out_dir, "decode_step.onnx"))
    files = sorted(f for f in os.listdir(out_dir) if f != "manifest.json")
    manifest = {"format_version": FORMAT_VERSION, "quantisation": "int4 per-row symmetric (q + 7 nibbles)",
                "files": {f: {"bytes": os.path.getsize(os.path.join(out_dir, f)), "sha256": _sha(os.path.join(out_dir, f))}
                          for f in files}}
    with open(os.path.join(out_dir, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)
    return manifest


def load_package(out_dir: str, device="cpu"):
    from ..config import ModelConfig
    from ..models.lm import build_model
    from ..quant.int4 import dequant_int4
    with open(os.path.join(out_dir, "manifest.json")) as f:
        man = json.load(f)
    for fname, meta in man["files"].items():
        if _sha(os.path.join(out_dir, fname)) != meta["sha256"]:
            raise ValueError(f"package file {fname} does not match its manifest")
    cfg = ModelConfig.from_dict(json.load(open(os.path.join(out_dir, "config.json"))))
    model = build_model(cfg, device=device, dtype=torch.float32)
    packed = torch.load(os.path.join(out_dir, "weights_int4.pt"))
    sd = {}
    for name, e in packed.items():
        if "int4" in e:
            sd[name] = dequant_int4(e["int4"], e["scale"], e["shape"][1])
        else:
            sd[name] = e["fp16"].float()
    model.load_state_dict(sd)
    return model
