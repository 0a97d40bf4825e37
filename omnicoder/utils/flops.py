"""Model FLOPs of a training step and model FLOPs utilisation (MFU).

FLOPs per trained token = 6 x (parameters a token multiplies: attention
projections, router, shared experts, top_k routed experts per MoE layer (dense
FFN for dense layers), output head; the embedding lookup is not a matmul)
+ attention scores and values: forward 2 x (S / 2) x heads x (Dq + Dv) per layer
for causal attention over S positions (S window-limited), times 3 for forward
+ backward.  Recomputation inside backward kernels is not counted (the usual
MFU convention).
"""
from __future__ import annotations


def _attn_dims(cfg):
    a = cfg.attn
    H = cfg.n_heads
    if a.kind == "mla":
        dq = a.qk_nope_dim + a.qk_rope_dim
        dv = a.v_head_dim
        q = cfg.d_model * H * dq
        kv_a = cfg.d_model * (a.kv_lora_rank + a.qk_rope_dim)
        kv_b = a.kv_lora_rank * H * (a.qk_nope_dim + a.v_head_dim)
        o = H * dv * cfg.d_model
        return H, dq, dv, q + kv_a + kv_b + o
    hd = a.head_dim or cfg.d_model // H
    hk = a.n_kv_heads or H
    return H, hd, hd, cfg.d_model * hd * (H + 2 * hk) + H * hd * cfg.d_model


def active_params_per_token(cfg) -> int:
    H, dq, dv, attn = _attn_dims(cfg)
    m = cfg.moe
    if m is not None and m.n_experts > 0:
        expert = 3 * cfg.d_model * m.ffn_dim
        ffn = m.top_k * expert + m.n_shared_experts * expert \
            + m.n_experts * cfg.d_model
    else:
        ffn = 3 * cfg.d_model * cfg.ffn_dim
    return cfg.n_layers * (attn + ffn) + cfg.vocab_size * cfg.d_model


def train_flops_per_token(cfg, seq_len: int) -> float:
    H, dq, dv, _ = _attn_dims(cfg)
    span = min(seq_len, cfg.attn.window) if cfg.attn.window else seq_len
    attn = 3 * cfg.n_layers * 2 * (span / 2) * H * (dq + dv)
    return 6.0 * active_params_per_token(cfg) + attn


def mfu(tokens_per_s: float, cfg, seq_len: int, n_gpus: int, peak_tflops: float) -> float:
    """Achieved model FLOP/s per GPU over `peak_tflops` (TFLOP/s per GPU)."""
    return tokens_per_s * train_flops_per_token(cfg, seq_len) / n_gpus / (peak_tflops * 1e12)
