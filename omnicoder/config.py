"""Typed configuration tree of omnicoder.

One dataclass per concern (model, MoE, attention, training, inference,
parallelism) and named presets.  Two families of presets exist:

* the reference's presets (``mobile_4gb``, ``mobile_2gb``, ``*_moe16``,
  ``draft_2b``, ``draft_3b``; src/omnicoder/config.py:4-58 and :113-187) with the
  same sizes, and
* the workload presets used for the B200 measurements: the tiny CPU parity
  model, the 2B-class MLA MoE pretraining model, the dense 20B GQA model, the
  long-context MoE inference model and its 2-layer draft model.

Environment variables never change a config; presets and explicit overrides
(``ModelConfig.replace``/CLI flags) do.
"""
from __future__ import annotations

import dataclasses
import json
import math
from dataclasses import dataclass, field
from typing import Any


@dataclass
class MoEConfig:
    """Routed experts of one MoE FFN layer."""

    n_experts: int = 0                  # 0 disables MoE (dense FFN)
    top_k: int = 2
    ffn_dim: int = 1408                 # per-expert hidden size
    n_shared_experts: int = 0           # always-on experts (DeepSeek style)
    capacity_factor: float = 0.0        # 0: dropless; else cap = ceil(cf * T * k / E)
    renorm_topk: bool = True            # renormalise the kept top-k probabilities
    aux_loss_alpha: float = 0.01        # load-balance loss weight
    z_loss_beta: float = 0.0            # router z-loss weight
    first_dense_layers: int = 0         # leading layers that use a dense FFN

    @property
    def enabled(self) -> bool:
        return self.n_experts > 0

    def capacity(self, tokens: int) -> int:
        if self.capacity_factor <= 0:
            return 0
        return int(math.ceil(self.capacity_factor * tokens * self.top_k / self.n_experts))


@dataclass
class AttentionConfig:
    """Self-attention variant and long-context knobs."""

    kind: str = "mha"                   # "mha" | "gqa" | "mla"
    n_kv_heads: int = 0                 # gqa: number of KV heads (0 = n_heads)
    head_dim: int = 0                   # mha/gqa: 0 = d_model // n_heads
    # MLA (latent KV): kv latent rank, rope part of q/k, nope part of q/k, v head dim
    kv_lora_rank: int = 512
    q_lora_rank: int = 0                # 0: direct q projection
    qk_rope_dim: int = 64
    qk_nope_dim: int = 128
    v_head_dim: int = 128
    # RoPE
    rope_theta: float = 10000.0
    rope_scale: float = 1.0             # positions are divided by this factor
    rope_interleaved: bool = False      # True: (2i, 2i+1) pairs as in the reference
    # long context
    window: int = 0                     # sliding window (0: full causal)
    mem_slots: int = 0                  # compressed memory slots visible to every query


@dataclass
class ModelConfig:
    """Decoder-only language model (spec family)."""

    name: str = "custom"
    vocab_size: int = 32000
    d_model: int = 256
    n_layers: int = 4
    n_heads: int = 8
    ffn_dim: int = 512                  # dense SwiGLU hidden size
    norm: str = "rmsnorm"               # "rmsnorm" | "layernorm"
    norm_eps: float = 1e-6
    tie_embeddings: bool = True
    max_seq_len: int = 4096
    init_std: float = 0.02
    mtp_heads: int = 0                  # extra next-next-token heads (speculative drafts)
    verifier_head: bool = False         # vocab-sized verifier head (speculative acceptance)
    attn: AttentionConfig = field(default_factory=AttentionConfig)
    moe: MoEConfig = field(default_factory=MoEConfig)

    # ------------------------------------------------------------------
    @property
    def head_dim(self) -> int:
        if self.attn.kind == "mla":
            return self.attn.qk_nope_dim + self.attn.qk_rope_dim
        return self.attn.head_dim or self.d_model // self.n_heads

    @property
    def n_kv_heads(self) -> int:
        if self.attn.kind == "gqa":
            return self.attn.n_kv_heads or self.n_heads
        return self.n_heads

    @property
    def v_head_dim(self) -> int:
        return self.attn.v_head_dim if self.attn.kind == "mla" else self.head_dim

    def is_moe_layer(self, i: int) -> bool:
        return self.moe.enabled and i >= self.moe.first_dense_layers

    def replace(self, **kw) -> "ModelConfig":
        return dataclasses.replace(self, **kw)

    def to_dict(self) -> dict[str, Any]:
        return dataclasses.asdict(self)

    @staticmethod
    def from_dict(d: dict[str, Any]) -> "ModelConfig":
        d = dict(d)
        attn = AttentionConfig(**d.pop("attn", {}))
        moe = MoEConfig(**d.pop("moe", {}))
        return ModelConfig(attn=attn, moe=moe, **d)

    def to_json(self) -> str:
        return json.dumps(self.to_dict(), indent=1, sort_keys=True)

    # ------------------------------------------------------------------
    def num_params(self, active_only: bool = False) -> int:
        """Parameter count from the shapes the model builds."""
        D, V = self.d_model, self.vocab_size
        n = V * D * (1 if self.tie_embeddings else 2) + D
        a = self.attn
        for i in range(self.n_layers):
            n += 2 * D
            if a.kind == "mla":
                qd = self.n_heads * (a.qk_nope_dim + a.qk_rope_dim)
                n += D * qd + D * (a.kv_lora_rank + a.qk_rope_dim) + a.kv_lora_rank
                n += a.kv_lora_rank * self.n_heads * (a.qk_nope_dim + a.v_head_dim)
                n += self.n_heads * a.v_head_dim * D
            else:
                hd = self.head_dim
                n += D * hd * (self.n_heads + 2 * self.n_kv_heads) + self.n_heads * hd * D
            if self.is_moe_layer(i):
                m = self.moe
                per = 3 * D * m.ffn_dim
                experts = m.top_k if active_only else m.n_experts
                n += D * m.n_experts + per * (experts + m.n_shared_experts)
            else:
                n += 3 * D * self.ffn_dim
        n += self.mtp_heads * D * V + (D * V if self.verifier_head else 0)
        return n


@dataclass
class TrainConfig:
    """Optimiser / schedule (reference TrainConfig, src/omnicoder/config.py:188-198)."""

    lr: float = 2e-4
    weight_decay: float = 0.01
    betas: tuple = (0.9, 0.95)
    eps: float = 1e-8
    warmup_steps: int = 1000
    max_steps: int = 100000
    grad_clip: float = 1.0
    micro_batch: int = 2
    seq_len: int = 4096
    grad_accum: int = 1
    seed: int = 0
    gradient_checkpointing: bool = False
    lora_r: int = 16
    lora_alpha: int = 32
    lora_dropout: float = 0.05


@dataclass
class ParallelConfig:
    """Process layout of one job: world = dp * tp * pp; EP groups live inside DP."""

    dp: int = 1
    ep: int = 1
    tp: int = 1
    pp: int = 1
    sequence_parallel: bool = False
    zero_stage: int = 1
    fp8: bool = False


@dataclass
class InferenceConfig:
    max_batch: int = 64
    max_new_tokens: int = 512
    kv_dtype: str = "bf16"              # "bf16" | "int8" | "int4"
    window: int = 0
    mem_slots: int = 0
    spec_tokens: int = 0                # draft proposals per step (0: no speculation)
    temperature: float = 0.0            # 0: greedy
    top_k: int = 0
    top_p: float = 1.0


@dataclass
class MultiModalConfig:
    """Unified vocabulary ranges (reference src/omnicoder/config.py:201-219)."""

    use_vision: bool = True
    use_video: bool = True
    use_audio: bool = True
    image_codebook_size: int = 8192
    video_codebook_size: int = 8192
    audio_codebook_size: int = 2048
    image_vocab_start: int = 32000
    video_vocab_start: int = 32000 + 8192
    audio_vocab_start: int = 32000 + 8192 + 8192


# ----------------------------------------------------------------------------
# Presets
# ----------------------------------------------------------------------------
def _tiny_moe() -> ModelConfig:
    # CPU parity model: 4 layers, d 256, 8 heads of 32, RoPE, RMSNorm, 4 SwiGLU
    # experts of ffn 512 with a top-2 softmax router, tied 32000 vocab.
    return ModelConfig(
        name="tiny_moe", vocab_size=32000, d_model=256, n_layers=4, n_heads=8, ffn_dim=512,
        tie_embeddings=True, max_seq_len=512,
        attn=AttentionConfig(kind="mha"),
        moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=512, renorm_topk=True, aux_loss_alpha=0.0),
    )


def _moe_mla_2b() -> ModelConfig:
    # MoE LM pretraining model: 24 layers, d 2048, 16-head MLA (kv latent 512,
    # rope 64), 32 routed experts of ffn 1408 (top-4) + 1 shared expert.
    return ModelConfig(
        name="moe_mla_24l", vocab_size=32000, d_model=2048, n_layers=24, n_heads=16, ffn_dim=1408,
        tie_embeddings=False, max_seq_len=4096,
        attn=AttentionConfig(kind="mla", kv_lora_rank=512, qk_rope_dim=64, qk_nope_dim=128, v_head_dim=128),
        moe=MoEConfig(n_experts=32, top_k=4, ffn_dim=1408, n_shared_experts=1, aux_loss_alpha=0.01),
    )


def _dense_20b() -> ModelConfig:
    # Dense ~20B: 48 layers, d 6144, 48 query / 8 KV heads of 128, SwiGLU 16384.
    return ModelConfig(
        name="dense_20b", vocab_size=32000, d_model=6144, n_layers=48, n_heads=48, ffn_dim=16384,
        tie_embeddings=False, max_seq_len=8192,
        attn=AttentionConfig(kind="gqa", n_kv_heads=8, head_dim=128),
    )


def _longctx_moe() -> ModelConfig:
    c = _moe_mla_2b()
    c.name = "longctx_moe"
    c.max_seq_len = 8192 + 512
    c.attn.window = 4096
    c.attn.mem_slots = 64
    return c


def _draft_2l() -> ModelConfig:
    return ModelConfig(
        name="draft_2l", vocab_size=32000, d_model=1024, n_layers=2, n_heads=8, ffn_dim=2816,
        tie_embeddings=True, max_seq_len=8192 + 512, attn=AttentionConfig(kind="mha"),
    )


def _reference_preset(name: str) -> ModelConfig:
    """Sizes of the reference's mobile/draft presets in the spec family's form."""
    n = name.lower().strip()
    table = {
        # name: (layers, d_model, heads, mlp, experts, top_k, kv_latent, max_seq)
        "mobile_4gb": (12, 1024, 8, 2816, 16, 2, 160, 8192),
        "mobile_2gb": (8, 768, 8, 2048, 8, 2, 128, 4096),
        "mobile_4gb_moe16": (12, 1024, 8, 2816, 16, 2, 160, 8192),
        "mobile_2gb_moe16": (8, 768, 8, 2048, 16, 2, 128, 4096),
        "draft_2b": (24, 2048, 16, 5504, 8, 2, 256, 8192),
        "draft_3b": (28, 2304, 18, 6144, 8, 2, 256, 8192),
    }
    if n not in table:
        raise KeyError(n)
    L, D, H, F, E, K, R, S = table[n]
    shared = 2 if n.endswith("moe16") else 1
    hd = D // H
    return ModelConfig(
        name=n, vocab_size=32000, d_model=D, n_layers=L, n_heads=H, ffn_dim=F, tie_embeddings=False,
        max_seq_len=S,
        attn=AttentionConfig(kind="mla", kv_lora_rank=R, qk_rope_dim=min(64, hd // 2),
                             qk_nope_dim=hd - min(64, hd // 2), v_head_dim=hd),
        moe=MoEConfig(n_experts=E, top_k=K, ffn_dim=F, n_shared_experts=shared, capacity_factor=1.2),
    )


PRESETS = {
    "tiny_moe": _tiny_moe,
    "moe_mla_24l": _moe_mla_2b,
    "dense_20b": _dense_20b,
    "longctx_moe": _longctx_moe,
    "draft_2l": _draft_2l,
}


def get_preset(name: str) -> ModelConfig:
    """Return a fresh ModelConfig for a named preset (workload or reference preset)."""
    if name in PRESETS:
        return PRESETS[name]()
    return _reference_preset(name)


def list_presets() -> list[str]:
    return sorted(PRESETS) + ["mobile_4gb", "mobile_2gb", "mobile_4gb_moe16", "mobile_2gb_moe16", "draft_2b",
                              "draft_3b"]


# Reference-compatible helpers -------------------------------------------------
def get_rope_scale_for_target_ctx(base_max_seq_len: int, target_ctx: int) -> float:
    """Position scale factor target/base for extending context (1.0 when not extending).

    Same contract as the reference helper (src/omnicoder/config.py:61-76).
    """
    if target_ctx <= 0 or target_ctx <= base_max_seq_len:
        return 1.0
    return float(target_ctx) / float(base_max_seq_len)


def get_rope_interp_base(base: float, scale: float, enabled: bool = False) -> float:
    """Base shrink by sqrt(scale) for position interpolation when `enabled` and scale > 1
    (reference src/omnicoder/config.py:78-94 reads the switch from the environment; here it
    is an argument)."""
    if not enabled or scale <= 1.0:
        return float(base)
    return float(base) / math.sqrt(scale)
