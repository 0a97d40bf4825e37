"""Hot ops of omnicoder.  Each op dispatches to the sm_100a extension when its
inputs live on a CUDA device and to a PyTorch implementation (the fp32 oracle)
on CPU."""
from .attention import attention, attention_kv, attention_torch
from .layers import (RopeTable, apply_rope, embedding, layer_norm, linear, linear_rope, rms_norm, split_norm,
                     swiglu_mlp)
from .loss import cross_entropy_logits, lm_head_cross_entropy
from .moe import cap_rows_for, moe_ffn, moe_ffn_torch, route_torch
from .optim import FusedAdamW, cosine_lr

__all__ = [
    "attention_kv", "split_norm",
    "attention", "attention_torch", "RopeTable", "apply_rope", "embedding", "layer_norm", "linear", "linear_rope", "rms_norm",
    "swiglu_mlp", "cross_entropy_logits", "lm_head_cross_entropy", "cap_rows_for", "moe_ffn", "moe_ffn_torch",
    "route_torch", "FusedAdamW", "cosine_lr",
]
