"""User-preference expert (reference src/omnicoder/tools/preference_expert_train.py:1-201): LoRA
adapters fine-tuned on a user's recent texts, and a small retrieval index over the same texts for
personalised retrieval at generation time.

  texts:   a folder of .txt / .md files or a JSONL of {"text": ...} rows
  train:   the model is frozen, LoRA adapters (rank r) go on its projections, and next-token cross
           entropy over windows of the tokenised texts trains only the adapters
  index:   the texts go into the product-quantised TF-IDF retriever (omnicoder.retrieval.pq), saved
           beside the adapters
  use:     `python -m omnicoder.inference.generate --pref_lora out/pref_lora.pt --pref_index out/index`
           loads the adapters onto the model and adds the top passages for the prompt to the
           retrieved texts
"""
from __future__ import annotations

import argparse
import json
import os

import torch

from .lora import inject_lora, lora_state_dict


def read_texts(path: str) -> list[str]:
    if os.path.isfile(path) and path.endswith(".jsonl"):
        with open(path, encoding="utf-8") as f:
            return [str(json.loads(ln).get("text", "")) for ln in f if ln.strip()]
    files = [path] if os.path.isfile(path) else sorted(
        os.path.join(r, f) for r, _, fs in os.walk(path) for f in fs if f.endswith((".txt", ".md")))
    out = []
    for fp in files:
        with open(fp, encoding="utf-8", errors="replace") as f:
            out.append(f.read())
    return [t for t in out if t.strip()]


def token_windows(texts: list[str], tok, seq_len: int) -> torch.Tensor:
    """[n, seq_len + 1] windows of the concatenated token stream (each text ends with EOS)."""
    stream = []
    for t in texts:
        stream += tok.encode(t) + [getattr(tok, "eos_id", 2)]
    n = max(1, (len(stream) - 1) // seq_len)
    stream += [0] * max(0, n * seq_len + 1 - len(stream))
    return torch.stack([torch.tensor(stream[i * seq_len:i * seq_len + seq_len + 1]) for i in range(n)])


def train_preference_lora(model, windows: torch.Tensor, steps: int, batch: int = 4, lr: float = 1e-3, r: int = 8,
                          alpha: int = 16, seed: int = 0) -> list[float]:
    inject_lora(model, r, alpha)
    opt = torch.optim.AdamW([p for p in model.parameters() if p.requires_grad], lr=lr)
    dev = next(model.parameters()).device
    g = torch.Generator().manual_seed(seed)
    losses = []
    for _ in range(steps):
        b = windows[torch.randint(0, len(windows), (min(batch, len(windows)),), generator=g)].to(dev)
        loss = model(b[:, :-1], labels=b[:, 1:])["loss"]
        opt.zero_grad(set_to_none=True)
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    return losses


def load_preference_lora(model, path: str) -> int:
    """Attach adapters of the saved rank and load their weights; returns the number loaded."""
    obj = torch.load(path, map_location="cpu", weights_only=True)
    inject_lora(model, int(obj["r"]), int(obj["alpha"]))
    missing = model.load_state_dict(obj["lora"], strict=False)
    unexpected = list(missing.unexpected_keys)
    if unexpected:
        raise ValueError(f"adapter weights do not fit this model: {unexpected[:3]}")
    return len(obj["lora"])


def main(argv=None):
    from ..config import get_preset
    from ..inference.builders import load_model
    from ..models.lm import build_model
    from ..retrieval.pq import PQRetriever
    from .checkpoint import _atomic_save
    from .tokenizer import get_tokenizer
    ap = argparse.ArgumentParser(description="LoRA preference expert + personal retrieval index")
    ap.add_argument("--data", required=True, help="folder of .txt / .md files or a JSONL of {text}")
    ap.add_argument("--ckpt", default="")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--seq_len", type=int, default=128)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--r", type=int, default=8)
    ap.add_argument("--alpha", type=int, default=16)
    ap.add_argument("--out_dir", default="weights/preference")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    texts = read_texts(a.data)
    if not texts:
        raise SystemExit(f"no texts under {a.data}")
    model = (load_model(a.ckpt, a.device, dtype=torch.float32)[0] if a.ckpt else
             build_model(get_preset(a.preset), a.device, dtype=torch.float32, seed=0))
    tok = get_tokenizer(model.cfg.vocab_size)
    losses = train_preference_lora(model, token_windows(texts, tok, a.seq_len), a.steps, a.batch, a.lr, a.r,
                                   a.alpha)
    os.makedirs(a.out_dir, exist_ok=True)
    _atomic_save({"lora": lora_state_dict(model), "r": a.r, "alpha": a.alpha}, os.path.join(a.out_dir, "pref_lora.pt"))
    PQRetriever(n_subspaces=4, n_centroids=min(16, len(texts))).fit(texts).save(os.path.join(a.out_dir, "index"))
    print(json.dumps({"texts": len(texts), "steps": a.steps, "first_loss": losses[0] if losses else None,
                      "last_loss": losses[-1] if losses else None, "out_dir": a.out_dir}))
    return 0


if __name__ == "__main__":
    main()
