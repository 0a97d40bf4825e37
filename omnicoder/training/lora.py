"""LoRA adapters (reference src/omnicoder/training/finetune_lora.py:16-210).

* `LoRALinear`: nn.Linear wrapper, y = x W^T + b + (alpha / r) * dropout(x) A B
  (A [in, r] Kaiming-uniform, B [r, out] zero), for module-based models (the
  compat family, Hugging Face teachers).
* Spec-family models keep raw weight tensors that the fused kernels consume;
  `inject_lora` puts a parametrisation on each targeted 2-D weight so that the
  kernels see W + (alpha / r) * (A B)^T (one [out, in] add per forward) while
  only A and B train.
* `merge_lora` folds the adapters into the weights; `lora_state_dict` returns
  only the adapter tensors.
"""
from __future__ import annotations

import argparse
import math

import torch
import torch.nn as nn
import torch.nn.utils.parametrize as P


class LoRALinear(nn.Module):
    def __init__(self, linear: nn.Linear, r: int = 16, alpha: int = 32, dropout: float = 0.0):
        super().__init__()
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.weight, self.bias = linear.weight, linear.bias
        self.weight.requires_grad_(False)
        self.r, self.scale = r, alpha / max(1, r)
        self.dropout = nn.Dropout(dropout) if dropout > 0 else nn.Identity()
        self.A = nn.Parameter(torch.empty(self.in_features, r, device=self.weight.device, dtype=self.weight.dtype))
        self.B = nn.Parameter(torch.zeros(r, self.out_features, device=self.weight.device, dtype=self.weight.dtype))
        nn.init.kaiming_uniform_(self.A, a=math.sqrt(5))

    def forward(self, x):
        return nn.functional.linear(x, self.weight, self.bias) + self.scale * (self.dropout(x) @ self.A @ self.B)


class LoRADelta(nn.Module):
    """Parametrisation W -> W + scale * (A B)^T for a raw [out, in] weight."""

    def __init__(self, out_f: int, in_f: int, r: int, alpha: int, device, dtype):
        super().__init__()
        self.scale = alpha / max(1, r)
        self.A = nn.Parameter(torch.empty(in_f, r, device=device, dtype=dtype))
        self.B = nn.Parameter(torch.zeros(r, out_f, device=device, dtype=dtype))
        nn.init.kaiming_uniform_(self.A, a=math.sqrt(5))

    def forward(self, W):
        return W + self.scale * (self.A @ self.B).t().to(W.dtype)


DEFAULT_TARGETS = ("wqkv", "wq", "wkv_a", "wkv_b", "wo", "w13", "w2")


def inject_lora(model: nn.Module, r: int = 16, alpha: int = 32, dropout: float = 0.0,
                targets: tuple = DEFAULT_TARGETS) -> int:
    """Freeze the model and attach adapters; returns the number of adapted weights."""
    for p in model.parameters():
        p.requires_grad_(False)
    n = 0
    for name, mod in list(model.named_modules()):
        for cname, child in list(mod.named_children()):
            if isinstance(child, nn.Linear):
                setattr(mod, cname, LoRALinear(child, r, alpha, dropout))
                n += 1
        for pname, p in list(mod.named_parameters(recurse=False)):
            if pname in targets and p.dim() == 2:
                P.register_parametrization(mod, pname, LoRADelta(p.shape[0], p.shape[1], r, alpha, p.device,
                                                                 torch.float32 if p.dtype == torch.bfloat16 else p.dtype))
                n += 1
    return n


@torch.no_grad()
def merge_lora(model: nn.Module) -> nn.Module:
    for mod in list(model.modules()):
        if P.is_parametrized(mod):
            for pname in list(mod.parametrizations.keys()):
                P.remove_parametrizations(mod, pname, leave_parametrized=True)
        for cname, child in list(mod.named_children()):
            if isinstance(child, LoRALinear):
                lin = nn.Linear(child.in_features, child.out_features, bias=child.bias is not None,
                                device=child.weight.device, dtype=child.weight.dtype)
                lin.weight.copy_(child.weight + child.scale * (child.A @ child.B).t())
                if child.bias is not None:
                    lin.bias.copy_(child.bias)
                setattr(mod, cname, lin)
    for p in model.parameters():
        p.requires_grad_(True)
    return model


def lora_state_dict(model: nn.Module) -> dict:
    return {k: v for k, v in model.state_dict().items() if k.endswith(".A") or k.endswith(".B")}


def main(argv=None):
    """Fine-tune a checkpoint with LoRA on a text folder / jsonl: only the adapters train."""
    ap = argparse.ArgumentParser()
    ap.add_argument("--ckpt", default=None)
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--data", default="synthetic")
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--seq_len", type=int, default=128)
    ap.add_argument("--batch_size", type=int, default=4)
    ap.add_argument("--lr", type=float, default=1e-3)
    ap.add_argument("--r", type=int, default=16)
    ap.add_argument("--alpha", type=int, default=32)
    ap.add_argument("--out", default="weights/lora.pt")
    ap.add_argument("--merge", action="store_true", help="save merged full weights instead of adapters")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    from ..config import get_preset
    from ..inference.builders import load_model
    from ..models.lm import build_model
    from .checkpoint import _atomic_save
    from .data import SyntheticTokens, TextFolderDataset, batches
    model = load_model(a.ckpt, a.device, dtype=torch.float32)[0] if a.ckpt else \
        build_model(get_preset(a.preset), a.device, dtype=torch.float32)
    n = inject_lora(model, a.r, a.alpha)
    opt = torch.optim.AdamW([p for p in model.parameters() if p.requires_grad], lr=a.lr)
    src = SyntheticTokens(model.cfg.vocab_size, a.seq_len) if a.data == "synthetic" else \
        TextFolderDataset(a.data, a.seq_len)
    it = batches(src, a.batch_size)
    for step in range(a.steps):
        ids, lab = next(it)
        loss = model(ids.to(a.device), labels=lab.to(a.device))["loss"]
        loss.backward()
        opt.step()
        opt.zero_grad()
        print(f"[lora] step {step + 1} loss {float(loss):.4f} ({n} adapted weights)", flush=True)
    if a.merge:
        merge_lora(model)
        _atomic_save({"model": model.state_dict(), "config": model.cfg.to_dict()}, a.out)
    else:
        _atomic_save({"lora": lora_state_dict(model), "r": a.r, "alpha": a.alpha}, a.out)


if __name__ == "__main__":
    main()
