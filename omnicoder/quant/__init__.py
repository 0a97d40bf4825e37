"""Quantisation: KV-cache schemes (int8 per-token/per-head symmetric, u8 / nf4
per-group), paged latent KV, int4 weight-only linear layers."""
from .int4 import Int4Linear, dequant_int4, matmul_int4, pack_int4, quantize_model_int4, register_int4_backend
from .kv import KvQuantMeta, PagedKvCache, dequantize_kv, quantize_kv

__all__ = ["Int4Linear", "dequant_int4", "matmul_int4", "pack_int4", "quantize_model_int4", "register_int4_backend",
           "KvQuantMeta", "PagedKvCache", "dequantize_kv", "quantize_kv"]
