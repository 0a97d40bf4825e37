"""Unified vocabulary layout (reference src/omnicoder/modeling/multimodal/vocab_map.py:12-169,
config.py:201-219): text ids [0, 32000), then image, video and audio codebooks
at fixed offsets (32000, 32000 + 8192, 32000 + 16384 by default).  The sidecar
(JSON) records the ranges next to a checkpoint; integrity checks reject
overlapping or out-of-order ranges."""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass

from ..config import MultiModalConfig


@dataclass
class VocabSidecar:
    text_range: list
    image_range: list
    video_range: list
    audio_range: list

    @staticmethod
    def from_config(cfg: MultiModalConfig | None = None, text_vocab: int = 32000) -> "VocabSidecar":
        c = cfg or MultiModalConfig()
        return VocabSidecar([0, text_vocab - 1],
                            [c.image_vocab_start, c.image_vocab_start + c.image_codebook_size - 1],
                            [c.video_vocab_start, c.video_vocab_start + c.video_codebook_size - 1],
                            [c.audio_vocab_start, c.audio_vocab_start + c.audio_codebook_size - 1])

    def integrity_checks(self) -> None:
        rs = [self.text_range, self.image_range, self.video_range, self.audio_range]
        for a, b in rs:
            if a < 0 or b < a:
                raise ValueError(f"bad range {(a, b)}")
        for (a0, b0), (a1, b1) in zip(rs, rs[1:]):
            if a1 <= b0:
                raise ValueError(f"overlapping vocabulary ranges {(a0, b0)} and {(a1, b1)}")

    @property
    def total(self) -> int:
        return self.audio_range[1] + 1

    def to_json(self) -> str:
        return json.dumps(asdict(self))

    def save(self, path: str) -> None:
        with open(path, "w") as f:
            f.write(self.to_json())

    @staticmethod
    def load(path: str) -> "VocabSidecar":
        with open(path) as f:
            return VocabSidecar(**json.load(f))

    def modality_of(self, token_id: int) -> str:
        for name in ("text", "image", "video", "audio"):
            a, b = getattr(self, f"{name}_range")
            if a <= token_id <= b:
                return name
        return "unknown"


def _start(layout, kind: str) -> int:
    if layout is None:
        layout = VocabSidecar.from_config()
    if isinstance(layout, VocabSidecar):
        return getattr(layout, f"{kind}_range")[0]
    return int(getattr(layout, f"{kind}_vocab_start"))


def map_image_tokens(codes, layout=None):
    s = _start(layout, "image")
    return [s + int(c) for c in codes]


def map_video_tokens(codes, layout=None):
    s = _start(layout, "video")
    return [s + int(c) for c in codes]


def map_audio_tokens(codes, layout=None):
    s = _start(layout, "audio")
    return [s + int(c) for c in codes]
