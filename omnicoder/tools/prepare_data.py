"""Tiny datasets for a fresh workspace: ``python -m omnicoder.tools.prepare_data --root data``
(reference src/omnicoder/tools/prepare_multimodal_data.py:1-182, which copies bundled samples into
place so that every trainer can run end to end).  Nothing is downloaded; the samples are generated:

  text/*.txt            short prose and code files            (pretrain / distill --data text/)
  code/tasks.jsonl      {prompt, target, tests}                (code-verify, multi_solution, rl)
  vl/images/*.pt        [3, S, S] images in [-1, 1]: coloured squares on a background
  vl/caption.jsonl      {image, caption}                        (vl_tasks --task caption)
  vl/vqa.jsonl          {image, question, answer}               (vl_tasks --task vqa)
  asr/*.pt, asr.jsonl   {audio, transcript}: tones named by pitch (vl_tasks --task asr)
  unified.jsonl         rows mixing the above                   (vl_tasks --task unified)
  marks.jsonl           {text, write, score}                    (write-threshold)
Every file is written only when it does not exist yet, so a rerun keeps edited data.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

_COLORS = {"red": (1.0, -1.0, -1.0), "green": (-1.0, 1.0, -1.0), "blue": (-1.0, -1.0, 1.0), "white": (1.0, 1.0, 1.0)}
_TEXTS = [
    "The cache keeps the keys and values of every earlier position, so each new token costs one row.",
    "A mixture of experts routes every token to a few feed-forward networks chosen by a small gate.",
    "def fibonacci(n):\n    a, b = 0, 1\n    for _ in range(n):\n        a, b = b, a + b\n    return a\n",
    "Gradient clipping scales the whole update when its norm exceeds the limit.",
]
_CODE = [
    ("Write add(a, b) returning the sum.", "def add(a, b):\n    return a + b\n",
     "from solution import add\n\ndef test_add():\n    assert add(2, 3) == 5\n"),
    ("Write is_even(n).", "def is_even(n):\n    return n % 2 == 0\n",
     "from solution import is_even\n\ndef test_even():\n    assert is_even(4) and not is_even(7)\n"),
    ("Write fact(n), the factorial.", "def fact(n):\n    r = 1\n    for i in range(2, n + 1):\n        r *= i\n    return r\n",
     "from solution import fact\n\ndef test_fact():\n    assert fact(5) == 120 and fact(0) == 1\n"),
]


def _write(path: str, text: str) -> bool:
    if os.path.exists(path):
        return False
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    with open(path, "w", encoding="utf-8") as f:
        f.write(text)
    return True


def _save(path: str, t: torch.Tensor) -> bool:
    if os.path.exists(path):
        return False
    os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
    torch.save(t, path)
    return True


def _jsonl(rows: list[dict]) -> str:
    return "".join(json.dumps(r) + "\n" for r in rows)


def square_image(color: str, size: int, pos: tuple[int, int], side: int) -> torch.Tensor:
    img = torch.full((3, size, size), -0.6)
    c = torch.tensor(_COLORS[color])[:, None, None]
    y, x = pos
    img[:, y:y + side, x:x + side] = c
    return img


def tone(freq: float, samples: int = 8000, sr: int = 16000) -> torch.Tensor:
    t = torch.arange(samples) / sr
    return 0.5 * torch.sin(2 * math.pi * freq * t)


def prepare(root: str, image_size: int = 32, n_images: int = 8) -> dict:
    made = []
    for i, t in enumerate(_TEXTS):
        if _write(os.path.join(root, "text", f"doc{i}.txt"), t):
            made.append(f"text/doc{i}.txt")
    if _write(os.path.join(root, "code", "tasks.jsonl"),
              _jsonl([{"prompt": p, "target": s, "tests": t} for p, s, t in _CODE])):
        made.append("code/tasks.jsonl")
    caps, vqa = [], []
    names = list(_COLORS)
    for i in range(n_images):
        color = names[i % len(names)]
        side = image_size // 4 + (i % 3) * (image_size // 8)
        pos = ((i * 5) % (image_size - side), (i * 3) % (image_size - side))
        rel = os.path.join("vl", "images", f"img{i}.pt")
        if _save(os.path.join(root, rel), square_image(color, image_size, pos, side)):
            made.append(rel)
        path = os.path.join(root, rel)
        size_word = ["small", "medium", "large"][i % 3]
        caps.append({"image": path, "caption": f"a {size_word} {color} square"})
        vqa.append({"image": path, "question": "what color is the square?", "answer": color})
    for name, rows in (("caption.jsonl", caps), ("vqa.jsonl", vqa)):
        if _write(os.path.join(root, "vl", name), _jsonl(rows)):
            made.append(f"vl/{name}")
    asr = []
    for i, f in enumerate((220, 330, 440, 550)):
        rel = os.path.join("asr", f"tone{i}.pt")
        if _save(os.path.join(root, rel), tone(f)):
            made.append(rel)
        asr.append({"audio": os.path.join(root, rel), "transcript": f"a tone at {f} hertz"})
    if _write(os.path.join(root, "asr", "asr.jsonl"), _jsonl(asr)):
        made.append("asr/asr.jsonl")
    unified = vqa[:2] + asr[:2] + [{"image": caps[2]["image"], "audio": asr[2]["audio"], "caption": caps[2]["caption"]},
                                   {"text": _TEXTS[0]}]
    if _write(os.path.join(root, "unified.jsonl"), _jsonl(unified)):
        made.append("unified.jsonl")
    marks = [{"text": t, "write": int(i % 2 == 0), "score": 0.8 if i % 2 == 0 else 0.2} for i, t in enumerate(_TEXTS)]
    if _write(os.path.join(root, "marks.jsonl"), _jsonl(marks)):
        made.append("marks.jsonl")
    return {"root": root, "written": made}


def main(argv=None):
    ap = argparse.ArgumentParser(description="generate tiny datasets for every trainer")
    ap.add_argument("--root", default="data")
    ap.add_argument("--image_size", type=int, default=32)
    ap.add_argument("--images", type=int, default=8)
    a = ap.parse_args(argv)
    r = prepare(a.root, a.image_size, a.images)
    print(json.dumps({"root": r["root"], "written": len(r["written"])}))
    return 0


if __name__ == "__main__":
    main()
