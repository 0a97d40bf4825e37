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
