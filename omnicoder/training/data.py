"""Training data.

* TextFolderDataset: every *.txt / *.md / *.py (configurable) file under a
  folder, tokenised once and concatenated into one token stream that is cut
  into (seq_len + 1)-token windows; each rank of a data-parallel job reads a
  disjoint, strided subset of windows (reference training/data/datamodule.py
  and pretrain.py:203-300 `_TextFolderDataset`).
* JsonlTextDataset: a "text" field per line (KD / SFT style corpora).
* SyntheticTokens: uniform random ids, deterministic in (seed, rank, step) --
  the benchmark workload.
* `batches()`: an infinite iterator of pinned (ids, labels) [B, S] pairs
  (labels = ids shifted by one) for the trainer.
"""
from __future__ import annotations

import glob
import json
import os
from typing import Iterator

import torch

from .tokenizer import get_tokenizer


class TokenStream:
    def __init__(self, tokens: torch.Tensor, seq_len: int, rank: int = 0, world: int = 1):
        self.tokens, self.seq_len = tokens, seq_len
        n = (tokens.numel() - 1) // seq_len
        if n <= 0:
            raise ValueError(f"corpus of {tokens.numel()} tokens is shorter than one window of {seq_len + 1}")
        self.windows = list(range(rank, n, world)) or [rank % n]

    def __len__(self):
        return len(self.windows)

    def __getitem__(self, i):
        s = self.windows[i % len(self.windows)] * self.seq_len
        w = self.tokens[s:s + self.seq_len + 1]
        return w[:-1], w[1:]


class TextFolderDataset(TokenStream):
    def __init__(self, root: str, seq_len: int, tokenizer=None, patterns=("*.txt", "*.md", "*.py"), rank: int = 0,
                 world: int = 1, max_files: int = 0):
        tok = tokenizer or get_tokenizer()
        files = []
        for p in patterns:
            files += glob.glob(os.path.join(root, "**", p), recursive=True)
        files = sorted(set(files))[: max_files or None]
        if not files:
            raise FileNotFoundError(f"no text files matching {patterns} under {root}")
        ids: list[int] = []
        for f in files:
            with open(f, encoding="utf-8", errors="replace") as fh:
                ids += tok.encode(fh.read()) + [getattr(tok, "eos_id", 2) or 2]
        super().__init__(torch.tensor(ids, dtype=torch.long), seq_len, rank, world)
        self.files = files


class JsonlTextDataset(TokenStream):
    def __init__(self, path: str, seq_len: int, tokenizer=None, field: str = "text", rank: int = 0, world: int = 1):
        tok = tokenizer or get_tokenizer()
        ids: list[int] = []
        with open(path, encoding="utf-8") as fh:
            for line in fh:
                line = line.strip()
                if line:
                    ids += tok.encode(str(json.loads(line).get(field, ""))) + [getattr(tok, "eos_id", 2) or 2]
        super().__init__(torch.tensor(ids, dtype=torch.long), seq_len, rank, world)


class SyntheticTokens:
    def __init__(self, vocab: int, seq_len: int, seed: int = 0, rank: int = 0):
        self.vocab, self.seq_len, self.seed, self.rank = vocab, seq_len, seed, rank

    def batch(self, batch: int, step: int):
        g = torch.Generator().manual_seed((self.seed * 1_000_003 + self.rank) * 1_000_003 + step)
        s = torch.randint(0, self.vocab, (batch, self.seq_len + 1), generator=g)
        return s[:, :-1].contiguous(), s[:, 1:].contiguous()


def batches(source, batch: int, shuffle_seed: int = 0, pin: bool = True) -> Iterator[tuple[torch.Tensor, torch.Tensor]]:
    step = 0
    if isinstance(source, SyntheticTokens):
        while True:
            ids, lab = source.batch(batch, step)
            step += 1
            yield (ids.pin_memory(), lab.pin_memory()) if pin and torch.cuda.is_available() else (ids, lab)
    g = torch.Generator().manual_seed(shuffle_seed)
    while True:
        order = torch.randperm(len(source), generator=g).tolist()
        for i in range(0, len(order) - batch + 1, batch):
            xs, ys = zip(*(source[j] for j in order[i:i + batch]))
            ids, lab = torch.stack(xs), torch.stack(ys)
            yield (ids.pin_memory(), lab.pin_memory()) if pin and torch.cuda.is_available() else (ids, lab)
        if len(order) < batch:
            xs, ys = zip(*(source[j % len(source)] for j in range(batch)))
            yield torch.stack(xs), torch.stack(ys)


# ----------------------------------------------------------------------------
# Data module with noise options, JSONL pair datasets, weighted mixture engine
# (reference src/omnicoder/training/data/*.py: DataModule, KD / VL / VQA JSONL
# datasets, DataEngine)
# ----------------------------------------------------------------------------
class DataModule:
    """Batches from a token source with optional input noise: `drop_p` replaces tokens by
    `mask_id`, `replace_p` by uniform random ids (labels keep the clean tokens)."""

    def __init__(self, source, batch: int, vocab: int, drop_p: float = 0.0, replace_p: float = 0.0,
                 mask_id: int = 0, seed: int = 0):
        self.it = batches(source, batch, shuffle_seed=seed, pin=False)
        self.vocab, self.drop_p, self.replace_p, self.mask_id = vocab, drop_p, replace_p, mask_id
        self.g = torch.Generator().manual_seed(seed)

    def __iter__(self):
        return self

    def __next__(self):
        ids, lab = next(self.it)
        if self.drop_p > 0 or self.replace_p > 0:
            ids = ids.clone()
            u = torch.rand(ids.shape, generator=self.g)
            ids[u < self.drop_p] = self.mask_id
            rep = (u >= self.drop_p) & (u < self.drop_p + self.replace_p)
            ids[rep] = torch.randint(0, self.vocab, (int(rep.sum()),), generator=self.g)
        return ids, lab


class JsonlPairs:
    """{"prompt": ..., "response": ...} lines (KD / SFT pairs) -> (ids, labels) with the prompt
    masked out of the labels; `tokenize(str) -> list[int]`."""

    def __init__(self, path: str, tokenize, seq_len: int, prompt_key: str = "prompt", response_key: str = "response"):
        import json
        self.items = []
        for line in open(path, encoding="utf-8"):
            line = line.strip()
            if not line:
                continue
            d = json.loads(line)
            p, r = tokenize(d[prompt_key]), tokenize(d[response_key])
            ids = (p + r)[:seq_len + 1]
            lab = ([-100] * len(p) + r)[:seq_len + 1]
            pad = seq_len + 1 - len(ids)
            self.items.append((torch.tensor(ids + [0] * pad), torch.tensor(lab + [-100] * pad)))

    def __len__(self):
        return len(self.items)

    def __getitem__(self, i):
        ids, lab = self.items[i]
        return ids[:-1], lab[1:]


class ImageTextJsonl:
    """{"image": path, "text": caption} lines -> (image tensor [3, S, S] in [-1, 1], token ids)."""

    def __init__(self, path: str, tokenize, image_size: int = 224, root: str | None = None):
        import json
        import os
        self.rows = [json.loads(l) for l in open(path, encoding="utf-8") if l.strip()]
        self.tok, self.size = tokenize, image_size
        self.root = root or os.path.dirname(os.path.abspath(path))

    def __len__(self):
        return len(self.rows)

    def __getitem__(self, i):
        import os

        import numpy as np
        from PIL import Image
        r = self.rows[i]
        img = Image.open(os.path.join(self.root, r["image"])).convert("RGB").resize((self.size, self.size))
        x = torch.from_numpy(np.asarray(img, dtype=np.float32) / 127.5 - 1.0).permute(2, 0, 1)
        return x, torch.tensor(self.tok(r["text"]))


class DataEngine:
    """Weighted mixture of iterators: each draw picks source i with probability w_i / sum(w)."""

    def __init__(self, sources: dict, weights: dict, seed: int = 0):
        self.names = list(sources)
        self.its = {k: iter(v) for k, v in sources.items()}
        w = torch.tensor([float(weights.get(k, 1.0)) for k in self.names])
        self.p = w / w.sum()
        self.g = torch.Generator().manual_seed(seed)
        self.counts = {k: 0 for k in self.names}

    def __iter__(self):
        return self

    def __next__(self):
        i = int(torch.multinomial(self.p, 1, generator=self.g))
        k = self.names[i]
        self.counts[k] += 1
        return k, next(self.its[k])
