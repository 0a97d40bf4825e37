"""Audio-visual synchronisation, open-vocabulary grounding / segmentation heads and the speech
adapters (reference src/omnicoder/modeling/multimodal/av_sync.py:8-80,
vision_grounding.py:7-134, asr.py:9-58, tts.py:7-83).

  AVSyncModule(d_audio, d_video, d_model, heads)(audio [B, Ta, da], video [B, Tv, dv])
      -> (audio-conditioned video features [B, min(Ta, Tv), d_model], alignment score [B, 1] in [0, 1])
      Both streams are projected to d_model; video queries attend to audio and audio queries to video;
      the score is (1 + cos) / 2 of the two attended streams, mean-pooled over the common length.
  RepRTAHead(d_model, num_props)(vision_tokens [B, T, C], text_embed [B, C]) -> (boxes [B, P, 4]
      as (cx, cy, w, h) in [0, 1], confidence logits [B, P])
      The text query is adapted with the pooled image tokens (the re-parameterised text-region
      alignment of YOLO-E style heads); token relevance is a softmax of scaled dot products.
      Proposals: the reference tiles one pooled feature P times; here proposal j pools the
      tokens around the j-th most relevant token (relevance x a Gaussian of the token-grid
      distance), so the P boxes differ.
  TextSegHead(d_model, grid_hw)(vision_tokens, text_embed=None) -> mask [B, 1, H, W] in [0, 1]
  ASRAdapter / TTSAdapter: faster-whisper / whisper and pyttsx3 backends when installed; each
      reports itself unavailable otherwise (nothing is downloaded).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F


class AVSyncModule(nn.Module):
    def __init__(self, d_audio: int, d_video: int, d_model: int = 512, num_heads: int = 4):
        super().__init__()
        d = max(32, int(d_model))
        self.d_model = d
        self.audio_proj = nn.Linear(d_audio, d, bias=False)
        self.video_proj = nn.Linear(d_video, d, bias=False)
        self.v_from_a = nn.MultiheadAttention(d, max(1, num_heads), batch_first=True)
        self.a_from_v = nn.MultiheadAttention(d, max(1, num_heads), batch_first=True)
        self.fuse = nn.Sequential(nn.LayerNorm(d), nn.Linear(d, d))

    def forward(self, audio: torch.Tensor, video: torch.Tensor):
        if audio.dim() != 3 or video.dim() != 3:
            raise ValueError("AVSyncModule expects [B, T, C] audio and video features")
        a, v = self.audio_proj(audio), self.video_proj(video)
        vf = self.fuse(self.v_from_a(v, a, a, need_weights=False)[0])
        af = self.a_from_v(a, v, v, need_weights=False)[0]
        n = min(af.shape[1], vf.shape[1])
        vf, af = vf[:, :n], af[:, :n]
        cos = (F.normalize(af.mean(1), dim=-1) * F.normalize(vf.mean(1), dim=-1)).sum(-1, keepdim=True)
        return vf, 0.5 * (cos + 1.0)


def _grid(T: int) -> tuple[int, int]:
    h = int(math.isqrt(T))
    while h > 1 and T % h:
        h -= 1
    return h, T // h


class RepRTAHead(nn.Module):
    def __init__(self, d_model: int = 384, num_props: int = 10, spread: float = 1.5):
        super().__init__()
        self.num_props, self.spread = num_props, spread
        self.token_proj = nn.Linear(d_model, d_model, bias=False)
        self.text_proj = nn.Linear(d_model, d_model, bias=False)
        self.adapter = nn.Sequential(nn.Linear(2 * d_model, d_model), nn.GELU(), nn.Linear(d_model, d_model))
        self.norm = nn.LayerNorm(d_model)
        self.bbox = nn.Linear(d_model, 4)
        self.conf = nn.Linear(d_model, 1)

    def forward(self, vision_tokens: torch.Tensor, text_embed: torch.Tensor):
        B, T, C = vision_tokens.shape
        vt = self.token_proj(vision_tokens)
        q = F.normalize(self.adapter(torch.cat([self.text_proj(text_embed), vision_tokens.mean(1)], -1)), dim=-1)
        rel = torch.softmax((vt * q[:, None]).sum(-1) / math.sqrt(C), -1)            # [B, T]
        P = min(self.num_props, T)
        centers = rel.topk(P, -1).indices                                             # [B, P]
        h, w = _grid(T)
        ys = torch.arange(T, device=vt.device) // w
        xs = torch.arange(T, device=vt.device) % w
        cy, cx = ys[centers], xs[centers]                                             # [B, P]
        d2 = (ys[None, None] - cy[..., None]) ** 2 + (xs[None, None] - cx[..., None]) ** 2
        wts = rel[:, None] * torch.exp(-d2.float() / (2 * self.spread ** 2))          # [B, P, T]
        wts = wts / wts.sum(-1, keepdim=True).clamp_min(1e-12)
        feat = self.norm(torch.einsum("bpt,btc->bpc", wts, vt))
        boxes = torch.sigmoid(self.bbox(feat))
        conf = self.conf(feat).squeeze(-1)
        if P < self.num_props:                                                        # fewer tokens than proposals
            boxes = F.pad(boxes, (0, 0, 0, self.num_props - P))
            conf = F.pad(conf, (0, self.num_props - P), value=float("-inf"))
        return boxes, conf


class TextSegHead(nn.Module):
    def __init__(self, d_model: int = 384, grid_hw: tuple[int, int] | None = None):
        super().__init__()
        self.proj = nn.Linear(d_model, 1)
        self.grid_hw = grid_hw

    def forward(self, vision_tokens: torch.Tensor, text_embed: torch.Tensor | None = None):
        B, T, C = vision_tokens.shape
        logits = self.proj(vision_tokens).squeeze(-1)
        if text_embed is not None:
            logits = logits + torch.softmax((vision_tokens * text_embed[:, None]).sum(-1) / math.sqrt(C), -1)
        h, w = self.grid_hw if self.grid_hw is not None else _grid(T)
        if h * w < T:
            logits = logits[:, :h * w]
        elif h * w > T:
            logits = F.pad(logits, (0, h * w - T), value=float("-inf"))
        return torch.sigmoid(logits.reshape(B, 1, h, w))


def _try_import(name: str):
    import importlib
    try:
        return importlib.import_module(name)
    except ImportError:
        return None


class ASRAdapter:
    """Speech to text with faster-whisper (preferred) or whisper, when installed and the model is
    available locally."""

    def __init__(self, model_size: str = "small"):
        self.model_size = model_size
        self.backend, self._model = None, None

    def available(self) -> bool:
        if self.backend is not None:
            return True
        fw = _try_import("faster_whisper")
        if fw is not None:
            try:
                self._model, self.backend = fw.WhisperModel(self.model_size, device="cpu"), "faster_whisper"
                return True
            except Exception:
                pass
        wh = _try_import("whisper")
        if wh is not None:
            try:
                self._model, self.backend = wh.load_model(self.model_size), "whisper"
                return True
            except Exception:
                pass
        return False

    def transcribe(self, audio) -> str:
        if not self.available():
            raise RuntimeError("no speech-recognition backend (faster-whisper / whisper) is available")
        if self.backend == "faster_whisper":
            segments, _ = self._model.transcribe(audio)
            return " ".join(s.text.strip() for s in segments)
        return self._model.transcribe(audio)["text"].strip()


class TTSAdapter:
    """Text to speech through pyttsx3 (offline) when installed."""

    def __init__(self):
        self.engine = None

    def available(self) -> bool:
        if self.engine is None:
            m = _try_import("pyttsx3")
            if m is None:
                return False
            try:
                self.engine = m.init()
            except Exception:
                return False
        return True

    def synthesize(self, text: str, path: str) -> str:
        if not self.available():
            raise RuntimeError("no text-to-speech backend (pyttsx3) is available")
        self.engine.save_to_file(text, path)
        self.engine.runAndWait()
        return path
