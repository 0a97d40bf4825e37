"""Multimodal front ends: unified vocabulary layout, modality composers, vision
backbone family (ViT / DINO-style / SigLIP-style / local transformers), patch
(vision) and mel (audio) encoders, vector quantiser, image / video / audio
VQ-VAEs and a mel vocoder, cross-modal aligners and grounding / segmentation
heads."""
from .vocab import VocabSidecar, map_audio_tokens, map_image_tokens, map_video_tokens
from .encoders import MelFrontend, PatchEncoder, VectorQuantizer
from .composer import FusionComposer, MultimodalComposer
from .backbones import VisionBackbone
from .vqvae import AudioVQ, ImageVQVAE, MelVocoder, VideoVQVAE
from .aligner import CrossModalVerifier, GroundingHead, PreAligner, SegmentationHead, av_offset, clip_loss

__all__ = ["VocabSidecar", "map_audio_tokens", "map_image_tokens", "map_video_tokens", "MelFrontend", "PatchEncoder",
           "VectorQuantizer", "MultimodalComposer", "FusionComposer", "VisionBackbone", "AudioVQ", "ImageVQVAE", "MelVocoder", "VideoVQVAE",
           "CrossModalVerifier", "GroundingHead", "PreAligner", "SegmentationHead", "av_offset", "clip_loss"]
