"""Inference utilities (reference src/omnicoder/inference/tool_use.py,
memory_estimator.py, unified.py, expert_branch_decode.py, multimodal_infer.py).

ToolRegistry: named tools; `run_calls(text)` finds `<tool>name(arg)</tool>`
spans in generated text, executes them (python code in the sandboxed child
process of the RL rewards, a safe arithmetic evaluator, user functions) and
splices `<result>...</result>` back in.
estimate_memory(cfg, ...): bytes of weights, KV cache (bf16 / int8 latent or
per-head), activations of a decode step, optimizer state for training.
UnifiedRouter: dispatches a request to the text / image / audio handler by
its declared modality (or by file extension of an attached path).
expert_branch_decode: generates candidates under different router top-k
settings of the MoE layers and keeps the one with the highest mean token
log-probability under the unmodified model.
"""
from __future__ import annotations

import ast
import operator
import re

import torch


# ---------------------------------------------------------------------------
_OPS = {ast.Add: operator.add, ast.Sub: operator.sub, ast.Mult: operator.mul, ast.Div: operator.truediv,
        ast.Pow: operator.pow, ast.Mod: operator.mod, ast.FloorDiv: operator.floordiv, ast.USub: operator.neg}


def safe_eval_arith(expr: str) -> float:
    def ev(n):
        if isinstance(n, ast.Expression):
            return ev(n.body)
        if isinstance(n, ast.Constant) and isinstance(n.value, (int, float)):
            return n.value
        if isinstance(n, ast.BinOp) and type(n.op) in _OPS:
            return _OPS[type(n.op)](ev(n.left), ev(n.right))
        if isinstance(n, ast.UnaryOp) and type(n.op) in _OPS:
            return _OPS[type(n.op)](ev(n.operand))
        raise ValueError(f"unsupported expression: {expr!r}")
    return ev(ast.parse(expr, mode="eval"))


class ToolRegistry:
    CALL = re.compile(r"<tool>\s*(\w+)\((.*?)\)\s*</tool>", re.S)

    def __init__(self):
        self.tools = {"calc": lambda a: str(safe_eval_arith(a)), "python": self._python}

    @staticmethod
    def _python(code: str) -> str:
        from ..training.rl import run_sandboxed
        rc, out = run_sandboxed(code, timeout_s=5.0)
        return out.strip() if rc == 0 else f"error({rc}): {out.strip()[-200:]}"

    def register(self, name: str, fn) -> None:
        self.tools[name] = fn

    def run_calls(self, text: str) -> str:
        def sub(m):
            name, arg = m.group(1), m.group(2).strip().strip("'\"")
            fn = self.tools.get(name)
            try:
                res = fn(arg) if fn is not None else f"unknown tool {name}"
            except Exception as e:  # a failing tool reports instead of raising
                res = f"error: {e}"
            return f"{m.group(0)}<result>{res}</result>"
        return self.CALL.sub(sub, text)


# ---------------------------------------------------------------------------
def estimate_memory(cfg, batch: int = 1, seq: int = 2048, kv_dtype: str = "bf16", training: bool = False,
                    param_bytes: int = 2) -> dict:
    D, L = cfg.d_model, cfg.n_layers
    n_params = 0
    n_params += cfg.vocab_size * D * (1 if cfg.tie_embeddings else 2)
    a = cfg.attn
    if a.kind == "mla":
        att = D * cfg.n_heads * (a.qk_nope_dim + a.qk_rope_dim) + D * (a.kv_lora_rank + a.qk_rope_dim) + \
            a.kv_lora_rank * cfg.n_heads * (a.qk_nope_dim + a.v_head_dim) + cfg.n_heads * a.v_head_dim * D
        kv_row = a.kv_lora_rank + a.qk_rope_dim
    else:
        hd = cfg.head_dim
        att = D * (cfg.n_heads + 2 * cfg.n_kv_heads) * hd + cfg.n_heads * hd * D
        kv_row = 2 * cfg.n_kv_heads * hd
    m = cfg.moe
    ffn = (3 * D * m.ffn_dim * (m.n_experts + m.n_shared_experts) + m.n_experts * D) if m.enabled else 3 * D * cfg.ffn_dim
    n_params += L * (att + ffn + 2 * D)
    kv_elem = 1 if kv_dtype == "int8" else 2
    kv = L * batch * seq * kv_row * kv_elem + (L * batch * seq * 4 * (1 if a.kind == "mla" else 2 * cfg.n_kv_heads)
                                                if kv_dtype == "int8" else 0)
    act = batch * D * 2 * 8 + batch * cfg.vocab_size * 4
    out = {"params": n_params, "weights_bytes": n_params * param_bytes, "kv_cache_bytes": kv,
           "decode_activation_bytes": act}
    if training:
        out["optimizer_bytes"] = n_params * (4 + 4 + 4 + 2)     # fp32 master, m, v + bf16 grad
        out["train_activation_bytes_estimate"] = L * batch * seq * D * 2 * 16
    out["total_bytes"] = sum(v for k, v in out.items() if k.endswith("_bytes"))
    return out


# ---------------------------------------------------------------------------
class UnifiedRouter:
    EXT = {".png": "image", ".jpg": "image", ".jpeg": "image", ".wav": "audio", ".flac": "audio", ".mp4": "video"}

    def __init__(self):
        self.handlers = {}

    def register(self, modality: str, fn) -> None:
        self.handlers[modality] = fn

    def __call__(self, request: dict):
        mod = request.get("modality")
        if mod is None and request.get("path"):
            import os
            mod = self.EXT.get(os.path.splitext(request["path"])[1].lower())
        mod = mod or "text"
        if mod not in self.handlers:
            raise KeyError(f"no handler for modality {mod!r}")
        return self.handlers[mod](request)


# ---------------------------------------------------------------------------
@torch.no_grad()
def expert_branch_decode(model, ids: torch.Tensor, max_new_tokens: int, top_ks=(1, 2), **gen_kw):
    """Candidates with the MoE layers' top-k changed to each value in `top_ks`; returns the
    candidate whose continuation has the highest mean log-probability under the original model."""
    from .generate import generate
    moes = [b.ffn for b in getattr(model, "blocks", []) if hasattr(getattr(b, "ffn", None), "cfg")
            and getattr(b.ffn.cfg, "moe", None) is not None and b.ffn.cfg.moe.enabled]
    orig = model.cfg.moe.top_k
    best, best_s = None, -float("inf")
    for k in top_ks:
        model.cfg.moe.top_k = k
        try:
            out = generate(model, ids, max_new_tokens, temperature=0.0, top_k=0, top_p=1.0, **gen_kw)
        finally:
            model.cfg.moe.top_k = orig
        seq = out if out.dim() == 2 else out[None]
        logits = model(seq[:, :-1], all_logits=True)["logits"].float()
        lp = torch.log_softmax(logits, -1).gather(-1, seq[:, 1:, None]).squeeze(-1)[:, ids.shape[-1] - 1:]
        s = float(lp.mean())
        if s > best_s:
            best, best_s = out, s
    del moes
    return best, best_s
