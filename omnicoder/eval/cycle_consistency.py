"""Cycle consistency of generated media (reference src/omnicoder/training/cycle_consistency.py:1-64:
caption the generated images and transcribe the generated audio, so the text can be compared with
the prompts that produced them).

For every image (.png / .jpg / .jpeg, or a saved .pt / .npy tensor) and audio file (.wav) in a
folder, a captioner and a transcriber turn the media back into text; when the
generating prompt is known (`prompts.jsonl` rows {"file", "prompt"} in the folder, or a `<file>.txt`
beside the file) the record also gets the agreement between that text and the prompt (the partial
ratio of omnicoder.eval.teacher_verify).  The reference uses BLIP and Whisper checkpoints; here the
captioner defaults to this package's vision-language model (a checkpoint saved by the
vision-language trainer, or random weights), and the transcriber is a caller-supplied callable
(speech-recognition weights are not bundled).  Output: one JSONL record per file and a summary with
the mean agreement per kind.
"""
from __future__ import annotations

import argparse
import json
import os
from typing import Callable

import torch

from .teacher_verify import partial_ratio

IMAGE_EXT = (".png", ".jpg", ".jpeg", ".pt", ".npy")
AUDIO_EXT = (".wav",)


def _prompts(media_dir: str) -> dict:
    out = {}
    p = os.path.join(media_dir, "prompts.jsonl")
    if os.path.exists(p):
        with open(p, encoding="utf-8") as f:
            for ln in f:
                if ln.strip():
                    r = json.loads(ln)
                    out[os.path.basename(r["file"])] = r["prompt"]
    return out


def cycle_records(media_dir: str, caption: Callable[[str], str] | None = None,
                  transcribe: Callable[[str], str] | None = None) -> tuple[list[dict], dict]:
    known = _prompts(media_dir)
    recs = []
    for fn in sorted(os.listdir(media_dir)):
        path = os.path.join(media_dir, fn)
        low = fn.lower()
        kind = ("image" if low.endswith(IMAGE_EXT) else "audio" if low.endswith(AUDIO_EXT) else None)
        if kind is None or not os.path.isfile(path):
            continue
        rec = {"file": path, "kind": kind}
        fn_text = caption if kind == "image" else transcribe
        key = "caption" if kind == "image" else "transcript"
        if fn_text is not None:
            try:
                rec[key] = fn_text(path)
            except Exception as e:    # one unreadable file is recorded, the sweep goes on
                rec["error"] = f"{type(e).__name__}: {e}"
        prompt = known.get(fn)
        side = os.path.splitext(path)[0] + ".txt"
        if prompt is None and os.path.exists(side):
            with open(side, encoding="utf-8") as f:
                prompt = f.read().strip()
        if prompt is not None:
            rec["prompt"] = prompt
            if key in rec:
                rec["agreement"] = partial_ratio(rec[key], prompt)
        recs.append(rec)
    summary = {}
    for kind in ("image", "audio"):
        sc = [r["agreement"] for r in recs if r["kind"] == kind and "agreement" in r]
        summary[kind] = {"files": sum(r["kind"] == kind for r in recs),
                         "mean_agreement": (sum(sc) / len(sc)) if sc else None}
    return recs, summary


def vl_captioner(ckpt: str = "", preset: str = "tiny_moe", image_size: int = 64, device: str = "cpu",
                 max_new_tokens: int = 16) -> Callable[[str], str]:
    """Greedy "Caption:" answers of this package's vision-language model."""
    from ..config import ModelConfig, get_preset
    from ..models.lm import build_model
    from ..multimodal.backbones import VisionBackbone
    from ..multimodal.composer import FusionComposer
    from ..training.tokenizer import get_tokenizer
    from ..training.vl_tasks import VLTaskTrainer, load_media
    obj = torch.load(ckpt, map_location="cpu", weights_only=False) if ckpt else {}
    cfg = ModelConfig.from_dict(obj["config"]) if "config" in obj else get_preset(preset)
    lm = build_model(cfg, device=device, dtype=torch.float32, seed=0).eval()
    comp = FusionComposer(cfg.d_model, vision=VisionBackbone("vit_tiny", image_size=image_size, depth=2)).to(device)
    if "model" in obj:
        lm.load_export_state_dict(obj["model"], strict=False)
    if "composer" in obj:
        comp.load_state_dict(obj["composer"], strict=False)
    tr = VLTaskTrainer(lm, comp.eval(), get_tokenizer(cfg.vocab_size), "caption", train_lm=False)
    return lambda path: tr.answer(load_media(path, image_size), "Caption:", max_new_tokens).strip()


def main(argv=None):
    ap = argparse.ArgumentParser(description="caption / transcribe generated media and compare with their prompts")
    ap.add_argument("--media_dir", required=True)
    ap.add_argument("--out", default="weights/cycle_consistency.jsonl")
    ap.add_argument("--vl_ckpt", default="", help="vision-language checkpoint used as the captioner")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--image_size", type=int, default=64)
    ap.add_argument("--device", default="cpu")
    a = ap.parse_args(argv)
    recs, summary = cycle_records(a.media_dir, vl_captioner(a.vl_ckpt, a.preset, a.image_size, a.device))
    os.makedirs(os.path.dirname(a.out) or ".", exist_ok=True)
    with open(a.out, "w", encoding="utf-8") as f:
        for r in recs:
            f.write(json.dumps(r) + "\n")
    print(json.dumps({"out": a.out, "summary": summary}))
    return 0


if __name__ == "__main__":
    main()
