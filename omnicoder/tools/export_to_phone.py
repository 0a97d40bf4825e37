"""Export a checkpoint for on-device use: ``python -m omnicoder.tools.export_to_phone``.

Reference: src/omnicoder/tools/export_to_phone.py:1-180 (export the decode step,
quantise, package and push to an Android / iOS device).  Here one command writes
a self-describing package directory:

  * int4 weight-only package (packed nibbles + per-row scales + manifest with
    checksums; omnicoder.export.mobile_packager) -- what the phone runtime loads;
  * GGUF file of the same weights (f16) for llama.cpp-style runtimes;
  * ONNX decode-step graph (and an optional prefill graph) when the `onnx`
    package is installed; otherwise the manifest records why it was skipped;
  * the decode step as a `torch.export` program and, when their packages are installed, its
    ExecuTorch (.pte) and Core ML conversions, plus an MLC compile recipe
    (omnicoder.export.mobile_runtimes);
  * a top-level `phone_manifest.json` with every artefact, its size and the
    model configuration.

Pushing to a device (adb / Xcode) is outside this container; `--push` prints the
adb commands for the package instead of running them.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time


def export_for_phone(model, out_dir: str, onnx: bool = True, prefill: int = 0, max_len: int = 512,
                     gguf: bool = True, runtimes: bool = True) -> dict:
    """Write the package; returns the manifest (also saved as phone_manifest.json)."""
    from ..export.gguf import export_model_gguf
    from ..export.mobile_packager import package_model
    os.makedirs(out_dir, exist_ok=True)
    man = {"created": time.strftime("%Y-%m-%dT%H:%M:%S"), "config": model.cfg.to_dict()
           if hasattr(model.cfg, "to_dict") else vars(model.cfg), "artifacts": {}}
    t0 = time.time()
    pkg = package_model(model, os.path.join(out_dir, "int4"))
    man["artifacts"]["int4_package"] = {"dir": "int4", "files": len(pkg["files"]),
                                        "bytes": sum(v["bytes"] for v in pkg["files"].values()),
                                        "seconds": round(time.time() - t0, 2)}
    if gguf:
        p = os.path.join(out_dir, "model.gguf")
        export_model_gguf(model, p)
        man["artifacts"]["gguf"] = {"file": "model.gguf", "bytes": os.path.getsize(p)}
    if onnx:
        from ..export.onnx_export import export_decode_step, export_prefill
        try:
            p = os.path.join(out_dir, "decode_step.onnx")
            export_decode_step(model, p, max_len=max_len)
            man["artifacts"]["onnx_decode_step"] = {"file": "decode_step.onnx", "bytes": os.path.getsize(p)}
            if prefill:
                p = os.path.join(out_dir, "prefill.onnx")
                export_prefill(model, p, prefill, max_len=max_len)
                man["artifacts"]["onnx_prefill"] = {"file": "prefill.onnx", "bytes": os.path.getsize(p)}
        except RuntimeError as e:
            man["artifacts"]["onnx_decode_step"] = {"skipped": str(e)}
    if runtimes:
        from ..export.mobile_runtimes import export_all
        try:
            man["artifacts"]["runtimes"] = export_all(model, os.path.join(out_dir, "runtimes"), max_len=max_len)
        except Exception as e:                 # an exporter limitation is reported, not fatal
            man["artifacts"]["runtimes"] = {"failed": f"{type(e).__name__}: {e}"}
    with open(os.path.join(out_dir, "phone_manifest.json"), "w") as f:
        json.dump(man, f, indent=1, default=str)
    return man


def adb_commands(out_dir: str, device_dir: str = "/sdcard/omnicoder") -> list[str]:
    return [f"adb shell mkdir -p {device_dir}", f"adb push {out_dir}/. {device_dir}/"]


def main(argv=None):
    ap = argparse.ArgumentParser(description="export a checkpoint as an on-device package")
    ap.add_argument("--ckpt", default="", help="checkpoint (default: random weights of --preset)")
    ap.add_argument("--preset", default="mobile_4gb")
    ap.add_argument("--out", default="weights/phone")
    ap.add_argument("--no_onnx", action="store_true")
    ap.add_argument("--no_gguf", action="store_true")
    ap.add_argument("--prefill", type=int, default=0, help="also export a prefill graph of this many tokens")
    ap.add_argument("--max_len", type=int, default=512)
    ap.add_argument("--push", action="store_true", help="print the adb commands that copy the package to a phone")
    a = ap.parse_args(argv)
    import torch
    if a.ckpt:
        from ..inference.builders import load_model
        model, _ = load_model(a.ckpt, "cpu", dtype=torch.float32, preset=a.preset)
    else:
        from ..inference.builders import build_mobile_model_by_name
        model = build_mobile_model_by_name(a.preset)
    man = export_for_phone(model.eval(), a.out, onnx=not a.no_onnx, prefill=a.prefill, max_len=a.max_len,
                           gguf=not a.no_gguf)
    print(json.dumps(man["artifacts"], indent=1, default=str))
    if a.push:
        print("\n".join(adb_commands(a.out)))
    return 0


if __name__ == "__main__":
    sys.exit(main())
