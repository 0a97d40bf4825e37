"""Modality composer (reference modeling/multimodal/fusion.py:64-681).

Builds one input sequence for the language model from text token embeddings
and other modalities, either as continuous features (projected to d_model and
wrapped in learned begin/end marker embeddings) or as discrete codes mapped into
the unified vocabulary (omnicoder.multimodal.vocab) and embedded by the LM's
own table.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from .vocab import VocabSidecar


class MultimodalComposer(nn.Module):
    MODALITIES = ("image", "video", "audio")

    def __init__(self, d_model: int, feature_dims: dict | None = None, layout: VocabSidecar | None = None):
        super().__init__()
        dims = feature_dims or {"image": d_model, "video": d_model, "audio": d_model}
        self.proj = nn.ModuleDict({m: nn.Linear(d, d_model) for m, d in dims.items()})
        self.bos = nn.ParameterDict({m: nn.Parameter(torch.randn(d_model) * 0.02) for m in dims})
        self.eos = nn.ParameterDict({m: nn.Parameter(torch.randn(d_model) * 0.02) for m in dims})
        self.layout = layout or VocabSidecar.from_config()

    def fuse_features(self, text_emb: torch.Tensor, **features: torch.Tensor) -> torch.Tensor:
        """text_emb [B, T, D]; features[m] [B, n_m, dim_m] -> [B, sum, D]: modalities first, then text."""
        parts = []
        B = text_emb.shape[0]
        for m in self.MODALITIES:
            f = features.get(m)
            if f is None:
                continue
            parts += [self.bos[m].expand(B, 1, -1), self.proj[m](f), self.eos[m].expand(B, 1, -1)]
        return torch.cat(parts + [text_emb], 1)

    def map_codes(self, codes: torch.Tensor, modality: str) -> torch.Tensor:
        return codes + getattr(self.layout, f"{modality}_range")[0]

    def fuse_codes(self, text_ids: torch.Tensor, **codes: torch.Tensor) -> torch.Tensor:
        """Token ids of a unified-vocabulary sequence: mapped modality codes, then text."""
        parts = [self.map_codes(c, m) for m, c in codes.items() if c is not None]
        return torch.cat(parts + [text_ids], 1)


def _feat_dim(enc, default: int) -> int:
    """Width of an encoder's output features."""
    for attr in ("dim", "out_dim"):
        if isinstance(getattr(enc, attr, None), int):
            return getattr(enc, attr)
    norm = getattr(enc, "norm", None)
    if isinstance(norm, nn.LayerNorm):
        return int(norm.normalized_shape[0])
    proj = getattr(enc, "proj", None)
    if isinstance(proj, nn.Linear):
        return proj.out_features
    if isinstance(proj, nn.Conv2d):
        return proj.out_channels
    return default


class FusionComposer(MultimodalComposer):
    """The full composer contract (reference modeling/multimodal/fusion.py:64-681) over this
    package's encoders, tokenizers and decoders; every component is optional and a method whose
    component is missing raises.

      encoders:  vision (VisionBackbone / PatchEncoder: image -> patch tokens), video
                 (VideoEncoder: frames -> per-frame features), audio (MelFrontend: wave ->
                 frame features) -- continuous inputs fused as projected features;
      tokenizers / decoders: image_vq, video_vq (VQ-VAEs), audio_vq (AudioVQ) and vocoder
                 (MelVocoder) -- discrete inputs mapped into the unified vocabulary, and
                 generated codes turned back into pixels / waveforms;
      heads:     grounding box and segmentation mask over image patches, audio-video offset.
    Segment ids of composed sequences: 0 text, 1 image, 2 video, 3 audio (markers included)."""

    SEGMENT = {"text": 0, "image": 1, "video": 2, "audio": 3}

    def __init__(self, d_model: int, vision=None, video=None, audio=None, image_vq=None, video_vq=None,
                 audio_vq=None, vocoder=None, layout: VocabSidecar | None = None):
        dims = {m: _feat_dim(enc, d_model) for m, enc in (("image", vision), ("video", video), ("audio", audio))
                if enc is not None}
        super().__init__(d_model, dims or {"image": d_model}, layout)
        self.vision, self.video_enc, self.audio_enc = vision, video, audio
        self.image_vq, self.video_vq, self.audio_vq, self.vocoder = image_vq, video_vq, audio_vq, vocoder
        from .aligner import GroundingHead, SegmentationHead
        self.ground = GroundingHead(d_model)
        self.seg = SegmentationHead(d_model)

    @staticmethod
    def _need(x, what: str):
        if x is None:
            raise RuntimeError(f"this composer was built without a {what}")
        return x

    # ---- continuous features -------------------------------------------------------------
    def image_tokens(self, image: torch.Tensor) -> torch.Tensor:
        out = self._need(self.vision, "vision encoder")(image)
        return out[0] if isinstance(out, tuple) else out

    def video_tokens(self, video: torch.Tensor) -> torch.Tensor:
        return self._need(self.video_enc, "video encoder")(video)[0]

    def audio_tokens(self, wav: torch.Tensor) -> torch.Tensor:
        return self._need(self.audio_enc, "audio encoder")(wav)

    def fuse_text_image(self, text_emb, image):
        return self.fuse_features(text_emb, image=self.image_tokens(image))

    def fuse_text_video(self, text_emb, video):
        return self.fuse_features(text_emb, video=self.video_tokens(video))

    def fuse_text_audio(self, text_emb, wav):
        return self.fuse_features(text_emb, audio=self.audio_tokens(wav))

    def fuse_all(self, text_emb, image=None, video=None, audio=None):
        """-> (embeddings [B, L, D], segment ids [B, L]) with modalities first, then text."""
        feats = {}
        if image is not None:
            feats["image"] = self.image_tokens(image)
        if video is not None:
            feats["video"] = self.video_tokens(video)
        if audio is not None:
            feats["audio"] = self.audio_tokens(audio)
        emb = self.fuse_features(text_emb, **feats)
        segs = []
        for m in self.MODALITIES:
            if m in feats:
                segs.append(torch.full((feats[m].shape[1] + 2,), self.SEGMENT[m], dtype=torch.long))
        segs.append(torch.zeros(text_emb.shape[1], dtype=torch.long))
        seg = torch.cat(segs).to(text_emb.device)[None].expand(text_emb.shape[0], -1)
        return emb, seg

    compose = fuse_all

    # ---- discrete codes --------------------------------------------------------------------
    def encode_image_to_codes(self, image):
        return self._need(self.image_vq, "image VQ-VAE").encode(image).flatten(1)

    def encode_video_to_codes(self, video):
        return self._need(self.video_vq, "video VQ-VAE").encode(video).flatten(1)

    def encode_audio_to_codes(self, wav):
        return self._need(self.audio_vq, "audio tokenizer").encode(wav)

    @staticmethod
    def map_codes_to_vocab(codes: torch.Tensor, offset: int) -> torch.Tensor:
        return codes + offset

    def fuse_text_image_codes(self, text_ids, image_codes):
        return self.fuse_codes(text_ids, image=image_codes)

    def fuse_text_video_codes(self, text_ids, video_codes):
        return self.fuse_codes(text_ids, video=video_codes)

    def fuse_text_audio_codes(self, text_ids, audio_codes):
        return self.fuse_codes(text_ids, audio=audio_codes)

    def decode_image_from_codes(self, codes, grid_shape: tuple[int, int]):
        vq = self._need(self.image_vq, "image VQ-VAE")
        return vq.decode(codes.view(codes.shape[0], *grid_shape))

    def decode_audio_from_codes(self, codes):
        mel = self._need(self.audio_vq, "audio tokenizer").decode(codes)
        return self._need(self.vocoder, "vocoder")(mel)

    # ---- heads ------------------------------------------------------------------------------
    def vision_heads(self, image_tokens, text_emb, image_size: int):
        """Grounding box (cx, cy, w, h in [0, 1]) of the text over the image, segmentation logits."""
        patches = self.proj["image"](image_tokens)
        grid = int(round(patches.shape[1] ** 0.5))
        return {"box": self.ground(text_emb, patches), "mask_logits": self.seg(patches, grid, image_size)}

    def video_heads(self, video_tokens):
        """Per-frame change score (1 - cosine of consecutive frame features) and the keyframe index."""
        f = torch.nn.functional.normalize(video_tokens, dim=-1)
        change = 1.0 - (f[:, 1:] * f[:, :-1]).sum(-1)
        return {"change": change, "keyframe": change.argmax(-1) + 1}

    def av_sync(self, audio_tokens, video_tokens, max_lag: int = 10):
        from .aligner import av_offset
        a, v = self.proj["audio"](audio_tokens), self.proj["video"](video_tokens)
        return {"offset": [av_offset(a[b], v[b], max_lag) for b in range(a.shape[0])]}

    def conditioning_from_hidden(self, hidden, segments=None):
        """Router conditioning: mean hidden state per modality present (zeros when absent)."""
        out = {}
        for m, sid in self.SEGMENT.items():
            if segments is None:
                out[m] = hidden.mean(1) if m == "text" else torch.zeros_like(hidden[:, 0])
                continue
            mask = (segments == sid).to(hidden.dtype)[..., None]
            out[m] = (hidden * mask).sum(1) / mask.sum(1).clamp_min(1.0)
        return out
