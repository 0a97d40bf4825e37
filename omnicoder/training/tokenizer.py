"""Tokenizers: a byte-level tokenizer that needs no files (the reference's
byte fallback, src/omnicoder/training/simple_tokenizer.py), and a wrapper for a
local Hugging Face tokenizer directory when one is provided."""
from __future__ import annotations

import os

PAD, BOS, EOS = 0, 1, 2
BYTE_OFFSET = 3


class ByteTokenizer:
    """UTF-8 bytes -> ids 3..258 (0 pad, 1 bos, 2 eos).  Works for any vocab >= 259."""

    def __init__(self, vocab_size: int = 32000):
        assert vocab_size >= 259
        self.vocab_size = vocab_size
        self.pad_id, self.bos_id, self.eos_id = PAD, BOS, EOS

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        ids = [b + BYTE_OFFSET for b in text.encode("utf-8")]
        return ([BOS] if add_bos else []) + ids

    def decode(self, ids) -> str:
        data = bytes(int(i) - BYTE_OFFSET for i in ids if BYTE_OFFSET <= int(i) < BYTE_OFFSET + 256)
        return data.decode("utf-8", errors="replace")


class HFTokenizer:
    def __init__(self, path: str):
        from transformers import AutoTokenizer

        self.tok = AutoTokenizer.from_pretrained(path, local_files_only=True)
        self.vocab_size = len(self.tok)
        self.eos_id = self.tok.eos_token_id

    def encode(self, text: str, add_bos: bool = False) -> list[int]:
        return self.tok.encode(text, add_special_tokens=add_bos)

    def decode(self, ids) -> str:
        return self.tok.decode(list(ids))


def get_tokenizer(vocab_size: int = 32000, path: str | None = None):
    path = path or os.environ.get("OMNICODER_TOKENIZER")
    if path and os.path.isdir(path):
        try:
            return HFTokenizer(path)
        except Exception as e:   # a broken tokenizer directory: say so, then use the byte tokenizer
            import warnings
            warnings.warn(f"tokenizer at {path} could not be loaded ({type(e).__name__}: {e}); "
                          f"using the byte tokenizer instead", RuntimeWarning, stacklevel=2)
    elif path:
        import warnings
        warnings.warn(f"tokenizer directory {path} does not exist; using the byte tokenizer", RuntimeWarning,
                      stacklevel=2)
    return ByteTokenizer(vocab_size)
