"""Multimodal front ends: unified vocabulary layout, modality composer, patch
(vision) and mel (audio) encoders, vector quantiser for discrete codes."""
from .vocab import VocabSidecar, map_audio_tokens, map_image_tokens, map_video_tokens
from .encoders import MelFrontend, PatchEncoder, VectorQuantizer
from .composer import MultimodalComposer

__all__ = ["VocabSidecar", "map_audio_tokens", "map_image_tokens", "map_video_tokens", "MelFrontend", "PatchEncoder",
           "VectorQuantizer", "MultimodalComposer"]
