"""Small operational tools behind one command: ``python -m omnicoder.tools.utilities <tool> ...``.

Each subcommand is the counterpart of one of the reference's single-purpose scripts
(src/omnicoder/tools/*.py):

  presets-export    model presets as JSON                         (presets_export.py:1-32)
  weights-validate  an exported package: files present, sizes and checksums match its manifests
                                                                  (weights_validator.py:1-31)
  threshold-check   fail when a metrics JSON's tokens/s is under a floor   (threshold_check.py:1-27)
  metrics-canary    measure decode tokens/s and write that metrics JSON    (metrics_canaries.py)
  kv-budget         KV bytes implied by a paging / quantisation sidecar against a limit
                                                                  (kv_budget_enforce.py:1-47)
  mobile-budget     artefact bytes of a package + KV bytes at a target context against a budget
                                                                  (mobile_budget_check.py:1-146)
  kv-calibrate      per-layer, per-group statistics of the KV cache over sample prompts and the
                    static u8 / nf4 parameters they imply                  (kv_calibrate.py:1-170)
  pq-build          product-quantised index over a folder of .txt files    (pq_build.py:1-45)
  router-ablate     decode tokens/s of the reference-layout MoE model with each router kind
                                                                  (router_ablate.py:1-77)
  env-audit         environment variables the package reads, documented-vs-used drift and the
                    set-but-unknown ones                                   (env_audit.py:1-92)
  gen-predictions   add a `prediction` to every row of a VQA / caption JSONL (gen_predictions.py)
  latent-refine     run a latent refiner checkpoint over a .npy of continuous image / audio latents
                                                                  (inference/mixed_latent_refine.py)
  act-calibrate     per-channel activation maxima of the GEMM inputs over sample prompts (prefill +
                    a few cached decode steps) and the static int8 scales they imply (act_calibrate.py)
  act-validate      check a calibration file (finite, positive scales) or print the effective knobs of
                    an activation-quantisation policy sidecar                 (validate_act_quant.py)
  kv-dump           the KV-cache rows of sample prompts, one .pt per prompt        (kv_dump.py)
  kv-autoencoder    a linear autoencoder of the dumped rows (closed-form PCA or AdamW) and its
                    sidecar                                                   (kv_autoencoder_train.py)
  kv-retention      the window / compressive-slot retention sidecar          (kv_retention_write.py)
  kv-prefetch       the pages-kept sidecar of the paged decode runner, capped at half the pages of a
                    paging sidecar                                           (kv_prefetch_write.py)
  code-verify       a solution against a pytest file in the sandbox, with pass / fail counts
                                                                  (code_verifier.py:1-97)
  auto-tune         the speculative draft length that maximises expected throughput, from a measured
                    acceptance benchmark                                       (auto_tune.py:1-138)
  plot-metrics      SVG charts written as text: bars of the numbers in a metrics JSON, lines of keys
                    of a JSONL training log                                  (visualize_metrics.py)
  write-threshold   the write-policy acceptance threshold per preset from teacher marks
                                                                  (write_policy_acceptance.py:1-103)

Exit codes follow the reference's scripts: 0 pass, 2 a checked limit was violated, 3 the input
could not be read.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import torch

GiB = 1 << 30
MiB = 1 << 20


def _write_json(path: str, obj) -> None:
    if not path:
        return
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    with open(path, "w", encoding="utf-8") as f:
        json.dump(obj, f, indent=1, default=str)


# ---- presets-export -------------------------------------------------------------
def presets_export(names: list[str] | None = None) -> dict:
    """{preset: ModelConfig as a dict} for the named presets (default: every preset)."""
    from ..config import get_preset, list_presets
    return {n: get_preset(n).to_dict() for n in (names or list_presets())}


def _cmd_presets_export(a) -> int:
    data = presets_export(a.names)
    _write_json(a.out, data)
    print(json.dumps({"presets": sorted(data), "out": a.out}))
    return 0


# ---- weights-validate -----------------------------------------------------------
def validate_package(root: str, required: tuple = ("phone_manifest.json",)) -> dict:
    """Check an exported package directory.

    * every `required` path exists;
    * every artefact `phone_manifest.json` lists with a `file` exists with the recorded size;
    * every sub-package with a `manifest.json` (the int4 package) has each listed file with the
      recorded size and sha256.
    Returns {"ok", "checked", "problems": [...]}.
    """
    from ..export.mobile_packager import _sha
    problems, checked = [], 0
    for rel in required:
        checked += 1
        if not os.path.exists(os.path.join(root, rel)):
            problems.append(f"missing: {rel}")
    top = os.path.join(root, "phone_manifest.json")
    if os.path.exists(top):
        with open(top, encoding="utf-8") as f:
            man = json.load(f)
        for name, art in man.get("artifacts", {}).items():
            if not isinstance(art, dict) or "file" not in art:
                continue
            checked += 1
            p = os.path.join(root, art["file"])
            if not os.path.exists(p):
                problems.append(f"{name}: missing {art['file']}")
            elif "bytes" in art and os.path.getsize(p) != art["bytes"]:
                problems.append(f"{name}: {art['file']} is {os.path.getsize(p)} bytes, manifest says {art['bytes']}")
    for d, _, files in os.walk(root):
        if "manifest.json" not in files:
            continue
        with open(os.path.join(d, "manifest.json"), encoding="utf-8") as f:
            sub = json.load(f)
        for fname, meta in sub.get("files", {}).items():
            checked += 1
            p = os.path.join(d, fname)
            rel = os.path.relpath(p, root)
            if not os.path.exists(p):
                problems.append(f"missing: {rel}")
            elif os.path.getsize(p) != meta.get("bytes", -1):
                problems.append(f"size mismatch: {rel}")
            elif "sha256" in meta and _sha(p) != meta["sha256"]:
                problems.append(f"checksum mismatch: {rel}")
    return {"ok": not problems, "checked": checked, "problems": problems}


def _cmd_weights_validate(a) -> int:
    r = validate_package(a.root, tuple(a.require))
    print(json.dumps(r))
    return 0 if r["ok"] else 2


# ---- metrics-canary / threshold-check -------------------------------------------
@torch.no_grad()
def decode_tokens_per_second(model, prompt_len: int = 32, new_tokens: int = 64, batch: int = 1,
                             kv_dtype: str = "bf16", warmup: int = 1) -> dict:
    """Greedy cached decode through the model's own cache path; tokens/s = batch * new_tokens / time."""
    from ..inference.kv_cache import KVCache
    dev = next(model.parameters()).device
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(1, model.cfg.vocab_size, (batch, prompt_len), generator=g).to(dev)

    def run():
        cache = KVCache(model.cfg, batch, prompt_len + new_tokens + 1, dev, kv_dtype=kv_dtype)
        logits = model.forward_cached(ids, cache, prefill=True, last_only=True)
        nxt = logits[:, -1].argmax(-1, keepdim=True)
        for _ in range(new_tokens - 1):
            nxt = model.forward_cached(nxt, cache, last_only=True)[:, -1].argmax(-1, keepdim=True)
        return nxt

    for _ in range(warmup):
        run()
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
    t0 = time.perf_counter()
    run()
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)
    dt = max(time.perf_counter() - t0, 1e-9)
    return {"tokens_per_second": batch * new_tokens / dt, "seconds": dt, "batch": batch,
            "new_tokens": new_tokens, "prompt_len": prompt_len, "kv_dtype": kv_dtype}


def _cmd_metrics_canary(a) -> int:
    from ..config import get_preset
    from ..models.lm import build_model
    dev = torch.device(a.device)
    dt = torch.float32 if dev.type == "cpu" else torch.bfloat16
    model = build_model(get_preset(a.preset), device=dev, dtype=dt, seed=0).eval()
    tok = decode_tokens_per_second(model, a.prompt_len, a.new_tokens, a.batch, a.kv_dtype)
    out = {"preset": a.preset, "device": str(dev), "tokens": tok}
    _write_json(a.out, out)
    print(json.dumps(out))
    return 0


def threshold_check(metrics_json: str, min_tps: float) -> tuple[int, str]:
    try:
        with open(metrics_json, encoding="utf-8") as f:
            tps = float(json.load(f).get("tokens", {}).get("tokens_per_second", 0.0))
    except (OSError, ValueError) as e:
        return 3, f"[threshold] ERROR: {e}"
    if tps < min_tps:
        return 2, f"[threshold] FAIL: tokens/s {tps:.2f} < {min_tps:.2f}"
    return 0, f"[threshold] OK: tokens/s {tps:.2f} >= {min_tps:.2f}"


def _cmd_threshold_check(a) -> int:
    code, msg = threshold_check(a.metrics_json, a.min_tps)
    print(msg)
    return code


# ---- kv-budget / mobile-budget --------------------------------------------------
def _prod(xs) -> int:
    n = 1
    for x in xs:
        n *= int(x)
    return n


def kv_bytes_from_sidecar(meta: dict, kvq: dict | None = None, elem_bytes: int = 2) -> int:
    """KV bytes one sequence needs, from a paging sidecar.

    This framework's sidecar carries the per-layer cache shapes (`k_shape`, `v_shape`, `n_layers`):
    bytes = n_layers * (|k| + |v|) * element bytes, or with a quantisation sidecar
    (`bits`, `group`) |kv| * bits / 8 plus one fp32 scale per group.  The reference's form
    (`page_len`, `heads`, `dl` or `dl_per_layer`, `spill_bytes`) is read as
    layers * heads * dl * page_len * 2 + spill_bytes.
    """
    if "k_shape" in meta:
        elems = int(meta.get("n_layers", 1)) * (_prod(meta["k_shape"]) + _prod(meta.get("v_shape", [0])))
        if kvq and kvq.get("bits"):
            return elems * int(kvq["bits"]) // 8 + -(-elems // max(1, int(kvq.get("group", 64)))) * 4
        return elems * elem_bytes
    page_len, heads = int(meta.get("page_len", 0)), int(meta.get("heads", 0))
    per_layer = meta.get("dl_per_layer")
    if isinstance(per_layer, list) and per_layer:
        kv = sum(int(d) for d in per_layer) * heads * page_len * 2
    else:
        kv = int(meta.get("n_layers", 0)) * heads * int(meta.get("dl", 0)) * page_len * 2
    return kv + max(0, int(meta.get("spill_bytes", 0)))


def _read_json(path: str) -> dict:
    with open(path, encoding="utf-8") as f:
        return json.load(f)


def _cmd_kv_budget(a) -> int:
    try:
        meta = _read_json(a.sidecar)
        kvq = _read_json(a.kvq_sidecar) if a.kvq_sidecar else None
    except (OSError, ValueError) as e:
        print(json.dumps({"error": str(e)}))
        return 3
    mb = kv_bytes_from_sidecar(meta, kvq) / MiB
    out = {"kv_mb": mb, "max_kv_mb": a.max_kv_mb, "pass": mb <= a.max_kv_mb, "source": a.sidecar}
    _write_json(a.out, out)
    print(json.dumps(out))
    return 0 if out["pass"] else 2


def kv_bytes_at(cfg, ctx: int, kvq: str = "bf16", group: int = 64, batch: int = 1) -> int:
    """KV bytes of `batch` sequences of `ctx` tokens: bf16; int8 as this framework stores it (one
    fp32 scale per latent row, or per head for GQA); u8 / nf4 with one fp32 scale per `group`."""
    a = cfg.attn
    if a.kind == "mla":
        per_tok, rows = a.kv_lora_rank + a.qk_rope_dim, 1
    else:
        per_tok, rows = 2 * cfg.n_kv_heads * cfg.head_dim, 2 * cfg.n_kv_heads
    n = cfg.n_layers * batch * ctx
    if kvq == "bf16":
        return n * per_tok * 2
    if kvq == "int8":
        return n * (per_tok + rows * 4)
    bits = {"u8": 8, "nf4": 4}[kvq]
    return n * (per_tok * bits // 8 + -(-per_tok // group) * 4)


def mobile_budget(root: str, target_ctx: int, kvq: str, budget_gb: float, preset: str | None = None) -> dict:
    """Resident memory of a package at `target_ctx` against `budget_gb`: the weights the runtime
    loads (the int4 package when present, else every file), the KV cache and the decode
    activations; also the package's total bytes on disk."""
    from ..config import ModelConfig, get_preset
    from ..inference.tools import estimate_memory
    disk = sum(os.path.getsize(os.path.join(d, f)) for d, _, fs in os.walk(root) for f in fs)
    int4 = os.path.join(root, "int4")
    weights = sum(os.path.getsize(os.path.join(int4, f)) for f in os.listdir(int4)) if os.path.isdir(int4) else disk
    man = os.path.join(root, "phone_manifest.json")
    if preset:
        cfg = get_preset(preset)
    elif os.path.exists(man):
        cfg = ModelConfig.from_dict(_read_json(man)["config"])
    else:
        raise ValueError("no phone_manifest.json in the package: pass a preset")
    kv = kv_bytes_at(cfg, target_ctx, kvq)
    act = estimate_memory(cfg, 1, target_ctx)["decode_activation_bytes"]
    total = weights + kv + act
    return {"disk_bytes": disk, "weights_bytes": weights, "kv_bytes": kv, "activation_bytes": act,
            "resident_bytes": total, "resident_gb": total / GiB, "budget_gb": budget_gb,
            "target_ctx": target_ctx, "kvq": kvq, "pass": total <= budget_gb * GiB}


def _cmd_mobile_budget(a) -> int:
    try:
        r = mobile_budget(a.release_root, a.target_ctx, a.kvq, a.budget_gb, a.preset)
    except (OSError, ValueError, KeyError) as e:
        print(json.dumps({"error": str(e)}))
        return 3
    bench = {}
    if a.bench_json and a.min_tps > 0:
        code, msg = threshold_check(a.bench_json, a.min_tps)
        bench = {"tps_check": msg, "tps_pass": code == 0}
        r["pass"] = r["pass"] and code == 0
    r.update(bench)
    _write_json(a.out, r)
    print(json.dumps(r))
    return 0 if r["pass"] else 2


# ---- kv-calibrate ---------------------------------------------------------------
_SAMPLE_PROMPTS = [
    "def fibonacci(n):\n    if n < 2:\n        return n\n    return fibonacci(n - 1) + fibonacci(n - 2)\n",
    "The quick brown fox jumps over the lazy dog while the compiler reports no warnings.",
    "SELECT name, count(*) FROM users GROUP BY name ORDER BY 2 DESC LIMIT 10;",
    "for (int i = 0; i < n; ++i) { acc += a[i] * b[i]; }",
]


class _GroupStats:
    """Running max / min / sum / sum of squares per (head, group) of one cache stream."""

    def __init__(self):
        self.mx = self.mn = self.s = self.ss = None
        self.n = 0

    def add(self, x: torch.Tensor, group: int):           # x [T, H, D]
        T, H, D = x.shape
        G = -(-D // group)
        x = torch.nn.functional.pad(x.float(), (0, G * group - D)).view(T, H, G, group)
        mx, mn = x.amax((0, 3)), x.amin((0, 3))
        s, ss = x.sum((0, 3)), (x * x).sum((0, 3))
        if self.mx is None:
            self.mx, self.mn, self.s, self.ss = mx, mn, s, ss
        else:
            self.mx, self.mn = torch.maximum(self.mx, mx), torch.minimum(self.mn, mn)
            self.s, self.ss = self.s + s, self.ss + ss
        self.n += T * group

    def params(self) -> dict:
        mean = self.s / max(1, self.n)
        std = (self.ss / max(1, self.n) - mean * mean).clamp_min(0).sqrt()
        scale = ((self.mx - self.mn) / 255.0).clamp_min(1e-8)
        return {"max": self.mx, "min": self.mn, "mean": mean, "std": std,
                "u8_scale": scale, "u8_zero": torch.round(-self.mn / scale).clamp(0, 255),
                "nf4_absmax": torch.maximum(self.mx.abs(), self.mn.abs())}


def _static_u8_error(x: torch.Tensor, p: dict, group: int) -> float:
    """Relative L2 error of quantising x [T, H, D] with the static u8 parameters."""
    T, H, D = x.shape
    G = p["u8_scale"].shape[-1]
    xp = torch.nn.functional.pad(x.float(), (0, G * group - D)).view(T, H, G, group)
    s, z = p["u8_scale"][None, :, :, None], p["u8_zero"][None, :, :, None]
    q = torch.clamp(torch.round(xp / s) + z, 0, 255)
    err = ((q - z) * s - xp).reshape(T, H, -1)[..., :D]
    return float(err.norm() / x.float().norm().clamp_min(1e-12))


@torch.no_grad()
def kv_calibrate(model, prompts: list[list[int]], group: int = 64) -> dict:
    """Run each prompt through the model's cached prefill and collect, per layer and per cache
    stream (MLA: the latent row; GQA: keys and values per head), statistics per group of `group`
    channels.  Returns {"group", "layers": [{stream: {stat: tensor [H, G]}}], "u8_rel_err": [...]}
    where u8_rel_err is the error of the static u8 parameters on the calibration data itself."""
    from ..inference.kv_cache import KVCache
    dev = next(model.parameters()).device
    L = model.cfg.n_layers
    stats = [dict() for _ in range(L)]
    seen = [[] for _ in range(L)]
    for ids in prompts:
        t = torch.tensor([ids], dtype=torch.long, device=dev)
        cache = KVCache(model.cfg, 1, len(ids) + 1, dev)
        model.forward_cached(t, cache, prefill=True, last_only=True)
        lo, hi = cache.sink, cache.sink + len(ids)
        for li in range(L):
            streams = {"k": cache.k[li][0, lo:hi]}
            if cache.v[li] is not None:
                streams["v"] = cache.v[li][0, lo:hi]
            for name, x in streams.items():
                x = x[:, None] if x.dim() == 2 else x          # MLA latent: one "head"
                stats[li].setdefault(name, _GroupStats()).add(x.cpu(), group)
            seen[li].append({k: (v[:, None] if v.dim() == 2 else v).cpu() for k, v in streams.items()})
    layers, errs = [], []
    for li in range(L):
        p = {name: st.params() for name, st in stats[li].items()}
        layers.append(p)
        e = [_static_u8_error(s[name], p[name], group) for s in seen[li] for name in s]
        errs.append(max(e) if e else 0.0)
    return {"group": group, "layers": layers, "u8_rel_err": errs}


def _cmd_kv_calibrate(a) -> int:
    from ..config import get_preset
    from ..inference.builders import load_model
    from ..models.lm import build_model
    from ..training.tokenizer import get_tokenizer
    dev = torch.device(a.device)
    model = (load_model(a.ckpt, dev, dtype=torch.float32)[0] if a.ckpt else
             build_model(get_preset(a.preset), device=dev, dtype=torch.float32, seed=0)).eval()
    tok = get_tokenizer(model.cfg.vocab_size)
    texts = _SAMPLE_PROMPTS
    if a.prompts:
        with open(a.prompts, encoding="utf-8") as f:
            texts = [ln.rstrip("\n") for ln in f if ln.strip()]
    ids = [tok.encode(t)[:a.max_tokens] or [1] for t in texts[:a.max_prompts or None]]
    r = kv_calibrate(model, ids, a.group)
    summary = {"scheme": a.scheme, "group": a.group, "prompts": len(ids), "layers": len(r["layers"]),
               "u8_rel_err_max": max(r["u8_rel_err"]),
               "per_layer": [{name: {"absmax": float(p[name]["nf4_absmax"].max()),
                                     "std_mean": float(p[name]["std"].mean())} for name in p}
                             for p in r["layers"]]}
    if a.scheme == "u8":
        summary["params"] = [{name: {"scale": p[name]["u8_scale"].tolist(), "zero": p[name]["u8_zero"].tolist()}
                              for name in p} for p in r["layers"]]
    else:
        summary["params"] = [{name: {"absmax": p[name]["nf4_absmax"].tolist(), "mean": p[name]["mean"].tolist(),
                                     "std": p[name]["std"].tolist()} for name in p} for p in r["layers"]]
    _write_json(a.out, summary)
    if a.stats_pt:
        torch.save(r, a.stats_pt)
    print(json.dumps({k: summary[k] for k in ("scheme", "group", "prompts", "layers", "u8_rel_err_max")}))
    return 0


# ---- pq-build ------------------------------------------------------------------
def pq_build(root: str, out_dir: str, m: int = 8, ks: int = 64, dim: int = 256, max_docs: int = 0) -> dict:
    """Index every .txt file under `root` (one document per file) and save it with a size profile."""
    from ..retrieval.pq import PQRetriever
    docs = []
    for d, _, files in sorted(os.walk(root)):
        for f in sorted(files):
            if f.endswith(".txt"):
                with open(os.path.join(d, f), encoding="utf-8", errors="replace") as fh:
                    docs.append(fh.read())
    if max_docs:
        docs = docs[:max_docs]
    if not docs:
        raise ValueError(f"no .txt files under {root}")
    pq = PQRetriever(m, ks, dim).fit(docs)
    pq.save(out_dir)
    prof = pq.budget_profile()
    _write_json(os.path.join(out_dir, "budget_profile.json"), prof)
    return prof


def _cmd_pq_build(a) -> int:
    try:
        prof = pq_build(a.root, a.out_dir, a.m, a.ks, a.dim, a.max_docs)
    except (OSError, ValueError) as e:
        print(json.dumps({"error": str(e)}))
        return 3
    print(json.dumps({"out_dir": a.out_dir, **prof}))
    return 0


# ---- router-ablate --------------------------------------------------------------
ROUTER_KINDS = ("topk", "multihead", "llm", "interaction", "hierarchical")


def _make_router(kind: str, D: int, E: int, k: int):
    from ..models import modules as M
    if kind == "topk":
        return M.TopKRouter(D, E, k=k)
    if kind == "multihead":
        return M.MultiHeadRouter(D, E, k=k, num_gates=4)
    if kind == "llm":
        return M.LLMRouter(D, E, k=k)
    if kind == "interaction":
        return M.InteractionRouter(D, E, k=k)
    if kind == "hierarchical":
        half = E // 2
        return M.HierarchicalRouter(D, E, group_sizes=[half, E - half], k=k)
    raise ValueError(f"router kind: one of {ROUTER_KINDS}")


@torch.no_grad()
def router_ablate(kinds=("topk", "llm"), new_tokens: int = 16, prompt_len: int = 8, device="cpu",
                  **compat_kw) -> dict:
    """Greedy decode tokens/s of the reference-layout model (models.compat.OmniTransformer, the
    layout whose MoE layers hold a swappable `router`) with every MoE layer's router replaced by
    each kind in turn; the same seed for every kind, so only the router differs."""
    from ..models.compat import OmniTransformer
    res = {}
    for kind in kinds:
        torch.manual_seed(0)
        model = OmniTransformer(**compat_kw).to(device).eval()
        c = model.c
        for blk in model.blocks:
            blk.moe.router = _make_router(kind, c.d_model, c.n_experts, c.top_k).to(device)
        ids = torch.randint(1, c.vocab_size, (1, prompt_len), generator=torch.Generator().manual_seed(0)).to(device)
        nxt, kv = model.decode_next_id(ids)                          # warm-up + first token
        t0 = time.perf_counter()
        for _ in range(new_tokens):
            nxt, kv = model.decode_next_id(nxt, kv)
        if str(device).startswith("cuda"):
            torch.cuda.synchronize()
        res[kind] = new_tokens / max(time.perf_counter() - t0, 1e-9)
    base = res.get(kinds[0], 0.0)
    return {"tokens_per_second": res, "baseline": kinds[0],
            "speedup_x": {k: v / max(base, 1e-9) for k, v in res.items()}, "new_tokens": new_tokens}


def _cmd_router_ablate(a) -> int:
    from ..config import get_preset
    kw = {}
    if a.preset:
        cfg = get_preset(a.preset)
        kw = dict(vocab_size=cfg.vocab_size, n_layers=cfg.n_layers, d_model=cfg.d_model, n_heads=cfg.n_heads,
                  mlp_dim=cfg.moe.ffn_dim if cfg.moe.enabled else cfg.ffn_dim,
                  n_experts=max(2, cfg.moe.n_experts if cfg.moe.enabled else 2), top_k=max(1, cfg.moe.top_k),
                  max_seq_len=cfg.max_seq_len, use_hrm=False)
    for key in ("n_layers", "d_model", "n_experts", "vocab_size"):
        if getattr(a, key):
            kw[key] = getattr(a, key)
    out = router_ablate(tuple(a.routers), a.max_new_tokens, device=a.device, **kw)
    out["config"] = kw
    _write_json(a.out_json, out)
    print(json.dumps(out))
    return 0


# ---- env-audit ------------------------------------------------------------------
def _documented_keys(path: str) -> list[str]:
    """KEY names of a KEY=VALUE example file (commented `# KEY=...` lines count as documented)."""
    keys = []
    if path and os.path.exists(path):
        with open(path, encoding="utf-8") as f:
            for line in f:
                s = line.strip().lstrip("#").strip()
                if "=" in s:
                    k = s.split("=", 1)[0].strip()
                    if k.replace("_", "").isalnum() and k.upper() == k:
                        keys.append(k)
    return sorted(set(keys))


def env_audit(root: str | None = None, env_example: str = "", prefix: str = "OMNICODER_") -> dict:
    """Variables read under `root`, the drift between them and an example file, and the variables
    with `prefix` that are set in this environment but read nowhere."""
    from ..utils.env import scan_registry
    reg = scan_registry(root)
    used = {k for k in reg if k.startswith(prefix)}
    doc = {k for k in _documented_keys(env_example) if k.startswith(prefix)}
    unknown = sorted(k for k in os.environ if k.startswith(prefix) and k not in reg)
    return {"registry": reg, "used_not_documented": sorted(used - doc),
            "documented_not_used": sorted(doc - used) if env_example else [], "unknown_set": unknown}


def _cmd_env_audit(a) -> int:
    from ..utils.env import load_dotenv, registry_markdown
    for p in (".env", ".env.tuned"):
        load_dotenv(p)
    r = env_audit(a.root or None, a.env_example, a.prefix)
    _write_json(a.out_json, r["registry"])
    if a.out_index:
        os.makedirs(os.path.dirname(a.out_index) or ".", exist_ok=True)
        with open(a.out_index, "w", encoding="utf-8") as f:
            f.write("# Environment variables read by the package\n\n" + registry_markdown(r["registry"]) + "\n")
    if a.sync_example and a.env_example:
        with open(a.env_example, "a", encoding="utf-8") as f:
            for k in r["used_not_documented"]:
                f.write(f"# {k}=\n")
    drift = bool(r["used_not_documented"] or r["documented_not_used"])
    print(json.dumps({"registry_count": len(r["registry"]), "used_not_documented": r["used_not_documented"],
                      "documented_not_used": r["documented_not_used"], "unknown_set": r["unknown_set"]}))
    return 1 if (a.fail_on_drift and drift and not a.sync_example) else 0


# ---- gen-predictions ------------------------------------------------------------
def gen_predictions(rows: list[dict], task: str, lm, composer, tokenizer, image_size: int = 64,
                    max_new_tokens: int = 16) -> list[dict]:
    """Each row with a `prediction`: VQA rows {image, question, ...}; caption rows {image, ...}."""
    from ..training.vl_tasks import TASKS, VLTaskTrainer, load_media
    name = {"vqa": "vqa", "captions": "caption", "caption": "caption"}[task]
    tr = VLTaskTrainer(lm, composer, tokenizer, name, train_lm=False)
    modality, template, _ = TASKS[name]
    out = []
    for r in rows:
        media = load_media(r[modality], image_size)
        prompt = template.format(question=r.get("question", ""))
        out.append({**r, "prediction": tr.answer(media, prompt, max_new_tokens).strip()})
    return out


def _cmd_gen_predictions(a) -> int:
    from ..config import ModelConfig, get_preset
    from ..models.lm import build_model
    from ..multimodal.backbones import VisionBackbone
    from ..multimodal.composer import FusionComposer
    from ..training.tokenizer import get_tokenizer
    dev = torch.device(a.device)
    obj = torch.load(a.ckpt, map_location="cpu", weights_only=False) if a.ckpt else {}
    cfg = ModelConfig.from_dict(obj["config"]) if "config" in obj else get_preset(a.preset)
    lm = build_model(cfg, device=dev, dtype=torch.float32, seed=0).eval()
    comp = FusionComposer(cfg.d_model, vision=VisionBackbone(a.vision, image_size=a.image_size, depth=2)).to(dev)
    if "model" in obj:
        lm.load_export_state_dict(obj["model"], strict=False)
    if "composer" in obj:
        comp.load_state_dict(obj["composer"], strict=False)
    with open(a.input, encoding="utf-8") as f:
        rows = [json.loads(ln) for ln in f if ln.strip()]
    if a.limit:
        rows = rows[:a.limit]
    preds = gen_predictions(rows, a.task, lm, comp.eval(), get_tokenizer(cfg.vocab_size), a.image_size,
                            a.max_new_tokens)
    os.makedirs(os.path.dirname(a.out) or ".", exist_ok=True)
    with open(a.out, "w", encoding="utf-8") as f:
        for r in preds:
            f.write(json.dumps(r) + "\n")
    print(json.dumps({"task": a.task, "rows": len(preds), "out": a.out}))
    return 0


# ---- latent-refine -------------------------------------------------------------
def latent_refine(latents, state: dict | None = None, hidden_mult: int = 2, temporal: bool = False):
    """[B, D] or [B, T, D] latents (numpy or tensor) through a LatentRefiner (weights from `state`,
    a state_dict, or the identity-initialised refiner when None); returns a float32 numpy array."""
    import numpy as np
    from ..multimodal.video import LatentRefiner
    x = torch.as_tensor(np.asarray(latents, dtype=np.float32))
    ref = LatentRefiner(x.shape[-1], hidden_mult=hidden_mult, temporal=temporal)
    if state is not None:
        ref.load_state_dict(state)
    else:                                 # no checkpoint: the residual branch off, latents pass through
        with torch.no_grad():
            ref.gate.zero_()
    with torch.no_grad():
        return ref.eval()(x).numpy()


def _cmd_latent_refine(a) -> int:
    import numpy as np
    state = None
    if a.ckpt:
        obj = torch.load(a.ckpt, map_location="cpu", weights_only=True)
        state = obj.get("refiner", obj) if isinstance(obj, dict) else obj
    out = latent_refine(np.load(a.latents), state, a.hidden_mult, a.temporal)
    np.save(a.out_latents, out)
    print(json.dumps({"in": a.latents, "out": a.out_latents, "shape": list(out.shape)}))
    return 0


# ---- act-calibrate / act-validate ----------------------------------------------
_ACT_MODULES = ("Norm", "LayerNorm", "Linear")     # outputs that are GEMM inputs (spec Norm; compat Linear)


@torch.no_grad()
def collect_activation_scales(model, prompts: list[list[int]], decode_steps: int = 8) -> dict:
    """{module name: per-channel max |activation| over the prompts} for the modules whose outputs
    feed the projections: RMSNorm / LayerNorm outputs of this package's model, Linear / LayerNorm
    outputs of the reference-layout model.  Each prompt runs a prefill and `decode_steps` greedy
    cached steps, so the decode path's activations count too."""
    stats: dict = {}

    def hook(name):
        def fn(_m, _inp, out):
            t = out if isinstance(out, torch.Tensor) else (out[0] if isinstance(out, (tuple, list)) else None)
            if not isinstance(t, torch.Tensor) or t.dim() == 0:
                return
            m = t.detach().float().abs().reshape(-1, t.shape[-1]).amax(0).cpu()
            stats[name] = torch.maximum(stats[name], m) if name in stats else m
        return fn

    hs = [m.register_forward_hook(hook(n)) for n, m in model.named_modules() if type(m).__name__ in _ACT_MODULES]
    dev = next(model.parameters()).device
    try:
        for ids in prompts:
            x = torch.tensor([ids], dtype=torch.long, device=dev)
            if hasattr(model, "forward_cached"):
                from ..inference.kv_cache import KVCache
                cache = KVCache(model.cfg, 1, len(ids) + decode_steps + 1, dev)
                nxt = model.forward_cached(x, cache, prefill=True, last_only=True)[:, -1].argmax(-1, keepdim=True)
                for _ in range(decode_steps):
                    nxt = model.forward_cached(nxt, cache, last_only=True)[:, -1].argmax(-1, keepdim=True)
            else:                                           # reference layout: prefill, then its decode path
                model(x)
                nxt, kv = model.decode_next_id(x)
                for _ in range(decode_steps):
                    nxt, kv = model.decode_next_id(nxt, kv)
    finally:
        for h in hs:
            h.remove()
    return stats


def _cmd_act_calibrate(a) -> int:
    from ..config import get_preset
    from ..inference.builders import load_model
    from ..models.lm import build_model
    from ..training.tokenizer import get_tokenizer
    dev = torch.device(a.device)
    model = (load_model(a.ckpt, dev, dtype=torch.float32)[0] if a.ckpt else
             build_model(get_preset(a.preset), device=dev, dtype=torch.float32, seed=0)).eval()
    tok = get_tokenizer(model.cfg.vocab_size)
    ids = [tok.encode(p)[:a.max_tokens] or [1] for p in (a.prompts or _SAMPLE_PROMPTS)]
    st = collect_activation_scales(model, ids, a.decode_steps)
    out = {"prompts": len(ids), "decode_steps": a.decode_steps,
           "modules": {k: {"absmax": v.tolist(), "int8_scale": (v.clamp_min(1e-8) / 127.0).tolist()}
                       for k, v in st.items()}}
    _write_json(a.out, out)
    print(json.dumps({"modules": len(st), "out": a.out,
                      "max_absmax": max((float(v.max()) for v in st.values()), default=0.0)}))
    return 0


def act_validate(obj: dict, layers: int = 0) -> dict:
    """A calibration file: every module's scales finite and positive, channel counts per module.
    A policy sidecar (the reference's *.act_quant.json: conf_floor, min_bits, max_bits, thresholds
    with layer_conf_floor or per-layer entries): the effective global and per-layer knobs."""
    import math
    if "modules" in obj:
        bad = [k for k, v in obj["modules"].items()
               if not v.get("int8_scale") or not all(math.isfinite(x) and x > 0 for x in v["int8_scale"])]
        return {"kind": "calibration", "modules": len(obj["modules"]), "bad": bad, "ok": not bad,
                "channels": sorted({len(v["int8_scale"]) for v in obj["modules"].values()})}
    floor = float(obj.get("conf_floor", 0.3))
    th = obj.get("thresholds", {}) if isinstance(obj.get("thresholds", {}), dict) else {}
    per = []
    if isinstance(th.get("layer_conf_floor"), (list, tuple)):
        per = [float(x) for x in th["layer_conf_floor"]]
    elif isinstance(th.get("layers"), dict):
        per = [float(v.get("conf_floor", floor)) for _, v in sorted((int(k), v) for k, v in th["layers"].items())]
    return {"kind": "policy", "ok": True,
            "global": {"conf_floor": floor, "min_bits": int(obj.get("min_bits", 8)),
                       "max_bits": int(obj.get("max_bits", 2))},
            "per_layer_conf_floor": per[:layers] if layers else per}


def _cmd_act_validate(a) -> int:
    try:
        obj = _read_json(a.policy)
    except (OSError, ValueError) as e:
        print(json.dumps({"error": str(e)}))
        return 3
    r = act_validate(obj, a.layers)
    print(json.dumps(r))
    return 0 if r["ok"] else 2


# ---- kv-dump / kv-autoencoder / kv-retention ------------------------------------
@torch.no_grad()
def kv_dump(model, prompts: list[list[int]], out_dir: str) -> list[str]:
    """One file per prompt: a list with, per layer, {"k": rows [T, ...], "v": rows or None} of the
    prompt's cache after prefill (MLA: the latent row; GQA: keys / values per head)."""
    from ..inference.kv_cache import KVCache
    os.makedirs(out_dir, exist_ok=True)
    dev = next(model.parameters()).device
    paths = []
    for i, ids in enumerate(prompts):
        cache = KVCache(model.cfg, 1, len(ids) + 1, dev)
        model.forward_cached(torch.tensor([ids], dtype=torch.long, device=dev), cache, prefill=True, last_only=True)
        lo, hi = cache.sink, cache.sink + len(ids)
        entry = [{"k": cache.k[li][0, lo:hi].float().cpu(),
                  "v": None if cache.v[li] is None else cache.v[li][0, lo:hi].float().cpu()}
                 for li in range(model.cfg.n_layers)]
        p = os.path.join(out_dir, f"kv_{i:05d}.pt")
        torch.save(entry, p)
        paths.append(p)
    return paths


class KVAutoEncoder(torch.nn.Module):
    def __init__(self, dim: int, latent: int):
        super().__init__()
        self.enc = torch.nn.Linear(dim, latent, bias=False)
        self.dec = torch.nn.Linear(latent, dim, bias=False)

    def forward(self, x):
        z = self.enc(x)
        return self.dec(z), z


def _kv_rows(kv_dir: str, max_files: int = 64) -> torch.Tensor:
    import glob
    rows = []
    for p in sorted(glob.glob(os.path.join(kv_dir, "kv_*.pt")))[:max_files]:
        for e in torch.load(p, map_location="cpu", weights_only=True):
            for t in (e["k"], e["v"]):
                if t is not None:
                    rows.append(t.reshape(-1, t.shape[-1]).float())
    return torch.cat(rows) if rows else torch.empty(0, 0)


def train_kv_autoencoder(rows: torch.Tensor, latent: int, method: str = "pca", steps: int = 500,
                         lr: float = 1e-3, seed: int = 0) -> tuple[KVAutoEncoder, float]:
    """Fit on rows [n, dim]; returns (model, relative reconstruction error on the rows).  `pca`: the
    optimal rank-`latent` linear autoencoder in closed form (encoder = top right singular vectors of
    the rows, decoder = its transpose); `sgd`: AdamW on the MSE from a random start."""
    n, dim = rows.shape
    ae = KVAutoEncoder(dim, min(latent, dim))
    if method == "pca":
        _, _, vh = torch.linalg.svd(rows, full_matrices=False)
        basis = vh[:ae.enc.out_features]                      # [latent, dim]
        with torch.no_grad():
            ae.enc.weight.copy_(basis)
            ae.dec.weight.copy_(basis.t())
    else:
        g = torch.Generator().manual_seed(seed)
        opt = torch.optim.AdamW(ae.parameters(), lr=lr)
        for _ in range(steps):
            xb = rows[torch.randint(0, n, (min(8192, n),), generator=g)]
            loss = torch.nn.functional.mse_loss(ae(xb)[0], xb)
            opt.zero_grad(set_to_none=True)
            loss.backward()
            torch.nn.utils.clip_grad_norm_(ae.parameters(), 1.0)
            opt.step()
    with torch.no_grad():
        err = float((ae(rows)[0] - rows).norm() / rows.norm().clamp_min(1e-12))
    return ae, err


def _cmd_kv_dump(a) -> int:
    from ..config import get_preset
    from ..inference.builders import load_model
    from ..models.lm import build_model
    from ..training.tokenizer import get_tokenizer
    dev = torch.device(a.device)
    model = (load_model(a.ckpt, dev, dtype=torch.float32)[0] if a.ckpt else
             build_model(get_preset(a.preset), device=dev, dtype=torch.float32, seed=0)).eval()
    tok = get_tokenizer(model.cfg.vocab_size)
    paths = kv_dump(model, [tok.encode(p)[:a.max_tokens] or [1] for p in (a.prompts or _SAMPLE_PROMPTS)], a.out_dir)
    print(json.dumps({"files": len(paths), "out_dir": a.out_dir}))
    return 0


def _cmd_kv_autoencoder(a) -> int:
    rows = _kv_rows(a.kv_dir)
    if rows.numel() == 0:
        print(json.dumps({"error": f"no kv_*.pt dumps in {a.kv_dir}"}))
        return 3
    ae, err = train_kv_autoencoder(rows, a.latent, a.method, a.steps, a.lr)
    os.makedirs(os.path.dirname(a.out_pt) or ".", exist_ok=True)
    torch.save({"dim": rows.shape[1], "latent": ae.enc.out_features, "state_dict": ae.state_dict()}, a.out_pt)
    side = {"kv_autoencoder": {"dim": rows.shape[1], "latent": ae.enc.out_features,
                               "weights": os.path.abspath(a.out_pt), "method": a.method, "rel_err": err}}
    _write_json(a.out_json, side)
    print(json.dumps(side["kv_autoencoder"]))
    return 0


def kv_prefetch(keep_pages: int, paging: dict | None = None) -> dict:
    keep = max(1, int(keep_pages))
    if paging:
        total = int(paging.get("total_pages", 0)) or int(paging.get("pages_per_layer", 0))
        if total > 0:
            keep = max(1, min(keep, total // 2))
    return {"keep_pages": keep}


def _cmd_kv_prefetch(a) -> int:
    out = kv_prefetch(a.keep_pages, _read_json(a.kv_paging_sidecar) if a.kv_paging_sidecar else None)
    _write_json(a.out, out)
    print(json.dumps(out))
    return 0


def _cmd_kv_retention(a) -> int:
    blob = {"compressive_slots": a.compressive_slots, "window_size": a.window_size, "schema": 1}
    _write_json(a.out, blob)
    print(json.dumps(blob))
    return 0


# ---- code-verify ---------------------------------------------------------------
def _cmd_code_verify(a) -> int:
    from ..sfb.sandbox import verify_with_tests
    if a.code_file:
        with open(a.code_file, encoding="utf-8") as f:
            code = f.read()
    else:
        code = a.code_text
    with open(a.tests_file, encoding="utf-8") as f:
        tests = f.read()
    name = os.path.basename(a.tests_file)
    r = verify_with_tests(code, tests, name if name.startswith("test_") else "test_" + name, a.timeout)
    out = {"ok": r.ok, "passed": r.passed, "failed": r.failed, "errors": r.errors, "returncode": r.returncode,
           "log": r.log}
    _write_json(a.out_json, out)
    print(json.dumps({k: v for k, v in out.items() if k != "log"}))
    return 0 if r.ok else 2


# ---- auto-tune -----------------------------------------------------------------
def expected_tokens(alpha: float, k: int) -> float:
    """Tokens per verification round with k drafts accepted independently with probability alpha:
    1 + alpha + ... + alpha^k (Leviathan et al., 2023)."""
    return float(k + 1) if alpha >= 1.0 else (1.0 - alpha ** (k + 1)) / (1.0 - alpha)


def alpha_from_ratio(ratio: float, k: int) -> float:
    """Per-token acceptance alpha from the measured accepted / proposed ratio of k-draft rounds:
    solves (alpha + alpha^2 + ... + alpha^k) / k = ratio by bisection (the ratio grows with alpha)."""
    ratio = min(max(ratio, 0.0), 1.0)
    lo, hi = 0.0, 1.0
    for _ in range(60):
        mid = 0.5 * (lo + hi)
        if (expected_tokens(mid, k) - 1.0) / k < ratio:
            lo = mid
        else:
            hi = mid
    return 0.5 * (lo + hi)


def tune_draft_len(report: dict, max_k: int = 16) -> dict:
    """From an acceptance benchmark (acceptance = accepted / proposed, draft_len k, plain and
    speculative tokens/s): per-token alpha, the draft-to-target step cost c implied by the measured
    speed-up (speculative / plain = E(k) / (k c + 1)), and the k in 1..max_k that maximises
    E(k) / (k c + 1); k = 0 (no drafting) when no k beats plain decoding."""
    r = report.get("acceptance", report)
    rep = r if isinstance(r, dict) else report          # nested (draft-pipeline report) or flat
    k0 = int(rep["draft_len"])
    alpha = alpha_from_ratio(float(rep["acceptance"]), k0)
    measured = float(rep["speculative_tokens_per_s"]) / max(float(rep["plain_tokens_per_s"]), 1e-9)
    c = max((expected_tokens(alpha, k0) / max(measured, 1e-9) - 1.0) / k0, 0.0)
    table = [{"draft_len": k, "expected_speedup": expected_tokens(alpha, k) / (k * c + 1.0)} for k in range(1, max_k + 1)]
    best = max(table, key=lambda t: t["expected_speedup"])
    k = best["draft_len"] if best["expected_speedup"] > 1.0 else 0
    return {"alpha": alpha, "cost_ratio": c, "measured_speedup": measured, "best_draft_len": k,
            "expected_speedup": best["expected_speedup"] if k else 1.0, "table": table,
            "generate_flags": f"--speculative_draft_len {k}" if k else "--disable_speculative"}


def _cmd_auto_tune(a) -> int:
    try:
        rep = _read_json(a.acceptance_json)
    except (OSError, ValueError) as e:
        print(json.dumps({"error": str(e)}))
        return 3
    out = tune_draft_len(rep, a.max_draft_len)
    _write_json(a.out, out)
    print(json.dumps({k: v for k, v in out.items() if k != "table"}))
    return 0


# ---- plot-metrics --------------------------------------------------------------
def _esc(t) -> str:
    return str(t).replace("&", "&amp;").replace("<", "&lt;").replace(">", "&gt;")


def svg_bars(data: dict, title: str = "", width: int = 640) -> str:
    """Horizontal bars, one per (label, value >= 0)."""
    items = [(k, max(0.0, float(v))) for k, v in data.items()]
    left, top, bar = 200, 30, 22
    height = top + bar * max(1, len(items)) + 10
    mx = max([v for _, v in items] + [1e-12])
    out = [f"<svg xmlns='http://www.w3.org/2000/svg' width='{width}' height='{height}'>",
           f"<text x='10' y='20' font-size='14' font-weight='bold'>{_esc(title)}</text>"]
    for i, (k, v) in enumerate(items):
        y = top + i * bar
        w = int((v / mx) * (width - left - 120))
        out.append(f"<text x='10' y='{y + 15}' font-size='12'>{_esc(k)[:28]}</text>")
        out.append(f"<rect x='{left}' y='{y + 2}' width='{w}' height='{bar - 6}' fill='#4C78A8'/>")
        out.append(f"<text x='{left + w + 6}' y='{y + 15}' font-size='12'>{v:.4g}</text>")
    out.append("</svg>")
    return "".join(out)


def svg_lines(series: dict, title: str = "", width: int = 640, height: int = 320) -> str:
    """One polyline per name of {name: [(x, y), ...]}, on shared axes."""
    pts = [p for ps in series.values() for p in ps]
    if not pts:
        return f"<svg xmlns='http://www.w3.org/2000/svg' width='{width}' height='60'><text x='10' y='30'>no data</text></svg>"
    x0, x1 = min(p[0] for p in pts), max(p[0] for p in pts)
    y0, y1 = min(p[1] for p in pts), max(p[1] for p in pts)
    sx = (width - 90) / ((x1 - x0) or 1.0)
    sy = (height - 70) / ((y1 - y0) or 1.0)
    colors = ["#4C78A8", "#F58518", "#54A24B", "#E45756", "#72B7B2", "#B279A2"]
    out = [f"<svg xmlns='http://www.w3.org/2000/svg' width='{width}' height='{height}'>",
           f"<text x='10' y='20' font-size='14' font-weight='bold'>{_esc(title)}</text>",
           f"<text x='10' y='{height - 30}' font-size='11'>{y0:.4g}</text><text x='10' y='45' font-size='11'>{y1:.4g}</text>",
           f"<text x='60' y='{height - 10}' font-size='11'>{x0:.4g}</text>"
           f"<text x='{width - 60}' y='{height - 10}' font-size='11'>{x1:.4g}</text>"]
    for i, (name, ps) in enumerate(series.items()):
        c = colors[i % len(colors)]
        path = " ".join(f"{60 + (x - x0) * sx:.1f},{height - 30 - (y - y0) * sy:.1f}" for x, y in ps)
        out.append(f"<polyline fill='none' stroke='{c}' stroke-width='1.5' points='{path}'/>")
        out.append(f"<text x='{width - 150}' y='{40 + 14 * i}' font-size='12' fill='{c}'>{_esc(name)}</text>")
    out.append("</svg>")
    return "".join(out)


def _numbers(obj, prefix: str = "") -> dict:
    out = {}
    if isinstance(obj, dict):
        for k, v in obj.items():
            out.update(_numbers(v, f"{prefix}{k}."))
    elif isinstance(obj, (int, float)) and not isinstance(obj, bool):
        out[prefix[:-1]] = float(obj)
    return out


def _cmd_plot_metrics(a) -> int:
    if a.log_jsonl:
        with open(a.log_jsonl, encoding="utf-8") as f:
            rows = [json.loads(ln) for ln in f if ln.strip()]
        keys = [k for k in a.keys.split(",") if k]
        series = {k: [(float(r.get(a.x, i)), float(r[k])) for i, r in enumerate(rows)
                      if isinstance(r.get(k), (int, float))] for k in keys}
        svg = svg_lines(series, a.title or os.path.basename(a.log_jsonl))
    else:
        nums = _numbers(_read_json(a.bench_json))
        if a.keys:
            nums = {k: v for k, v in nums.items() if any(s in k for s in a.keys.split(","))}
        svg = svg_bars(nums, a.title or os.path.basename(a.bench_json))
    os.makedirs(os.path.dirname(a.out_svg) or ".", exist_ok=True)
    with open(a.out_svg, "w", encoding="utf-8") as f:
        f.write(svg)
    print(json.dumps({"out_svg": a.out_svg}))
    return 0


# ---- write-threshold -------------------------------------------------------------
def write_threshold(marks: list[dict]) -> dict:
    """Marks {"write": 0 | 1, optional "score": the write head's probability}.  Without scores the
    threshold is the teacher's acceptance rate (the reference's fallback).  With scores it is the
    score quantile that accepts that same fraction of rows, and the F1-best threshold is reported
    beside it."""
    y = [int(m["write"]) for m in marks if "write" in m]
    rate = sum(y) / len(y) if y else 0.5
    scored = [(float(m["score"]), int(m["write"])) for m in marks if "score" in m and "write" in m]
    if not scored:
        return {"threshold": rate, "acceptance_rate": rate, "rows": len(y), "from": "labels"}
    sc = sorted((s for s, _ in scored), reverse=True)
    n_acc = round(rate * len(sc))
    thr = sc[n_acc - 1] if n_acc > 0 else sc[0] + 1e-6
    best = (0.0, thr)
    for t in sorted(set(sc)):
        tp = sum(1 for s, l in scored if s >= t and l)
        fp = sum(1 for s, l in scored if s >= t and not l)
        fn = sum(1 for s, l in scored if s < t and l)
        f1 = 2 * tp / max(1, 2 * tp + fp + fn)
        if f1 > best[0]:
            best = (f1, t)
    return {"threshold": thr, "acceptance_rate": rate, "rows": len(scored), "from": "scores",
            "f1_best_threshold": best[1], "f1": best[0]}


def _cmd_write_threshold(a) -> int:
    with open(a.marks, encoding="utf-8") as f:
        marks = [json.loads(ln) for ln in f if ln.strip()]
    r = write_threshold(marks)
    data = _read_json(a.out) if os.path.exists(a.out) else {}
    data[a.preset] = r["threshold"]
    _write_json(a.out, data)
    print(json.dumps({"preset": a.preset, **r, "out": a.out}))
    return 0


# ---- command line ---------------------------------------------------------------
def _parser() -> argparse.ArgumentParser:
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    ap = argparse.ArgumentParser(description="omnicoder operational tools")
    sub = ap.add_subparsers(dest="tool", required=True)

    p = sub.add_parser("presets-export", help="model presets as JSON")
    p.add_argument("--out", default="weights/presets.json")
    p.add_argument("--names", nargs="*", default=None)
    p.set_defaults(fn=_cmd_presets_export)

    p = sub.add_parser("weights-validate", help="check an exported package against its manifests")
    p.add_argument("--root", default="weights/phone")
    p.add_argument("--require", nargs="*", default=["phone_manifest.json"])
    p.set_defaults(fn=_cmd_weights_validate)

    p = sub.add_parser("threshold-check", help="fail when tokens/s is under a floor")
    p.add_argument("--metrics_json", default="weights/metrics_canaries.json")
    p.add_argument("--min_tps", type=float, default=20.0)
    p.set_defaults(fn=_cmd_threshold_check)

    p = sub.add_parser("metrics-canary", help="measure cached-decode tokens/s")
    p.add_argument("--preset", default="tiny_moe")
    p.add_argument("--prompt_len", type=int, default=32)
    p.add_argument("--new_tokens", type=int, default=64)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--kv_dtype", default="bf16", choices=["bf16", "int8"])
    p.add_argument("--out", default="weights/metrics_canaries.json")
    p.add_argument("--device", default=dev)
    p.set_defaults(fn=_cmd_metrics_canary)

    p = sub.add_parser("kv-budget", help="KV bytes of a paging sidecar against a limit")
    p.add_argument("--sidecar", required=True)
    p.add_argument("--kvq_sidecar", default="")
    p.add_argument("--max_kv_mb", type=float, default=1024.0)
    p.add_argument("--out", default="weights/kv_budget_summary.json")
    p.set_defaults(fn=_cmd_kv_budget)

    p = sub.add_parser("mobile-budget", help="resident bytes of a package at a target context")
    p.add_argument("--release_root", default="weights/phone")
    p.add_argument("--target_ctx", type=int, default=8192)
    p.add_argument("--kvq", default="int8", choices=["bf16", "int8", "u8", "nf4"])
    p.add_argument("--budget_gb", type=float, default=4.0)
    p.add_argument("--preset", default=None, help="model config (default: the package's manifest)")
    p.add_argument("--bench_json", default="", help="metrics JSON whose tokens/s must reach --min_tps")
    p.add_argument("--min_tps", type=float, default=0.0)
    p.add_argument("--out", default="weights/mobile_budget.json")
    p.set_defaults(fn=_cmd_mobile_budget)

    p = sub.add_parser("kv-calibrate", help="KV-cache statistics and static quantisation parameters")
    p.add_argument("--preset", default="tiny_moe")
    p.add_argument("--ckpt", default="")
    p.add_argument("--prompts", default="", help="text file, one prompt per line (default: built-in samples)")
    p.add_argument("--max_prompts", type=int, default=0)
    p.add_argument("--max_tokens", type=int, default=512)
    p.add_argument("--group", type=int, default=64)
    p.add_argument("--scheme", default="u8", choices=["u8", "nf4"])
    p.add_argument("--out", default="weights/kvq_calibration.json")
    p.add_argument("--stats_pt", default="", help="also save the raw statistics tensors here")
    p.add_argument("--device", default="cpu")
    p.set_defaults(fn=_cmd_kv_calibrate)

    p = sub.add_parser("pq-build", help="product-quantised index over a folder of .txt files")
    p.add_argument("root")
    p.add_argument("out_dir")
    p.add_argument("--m", type=int, default=8)
    p.add_argument("--ks", type=int, default=64)
    p.add_argument("--dim", type=int, default=256)
    p.add_argument("--max_docs", type=int, default=0)
    p.set_defaults(fn=_cmd_pq_build)

    p = sub.add_parser("router-ablate", help="decode tokens/s per router kind")
    p.add_argument("--preset", default="", help="sizes of this preset (default: the compat defaults)")
    p.add_argument("--routers", nargs="+", default=["topk", "llm"], choices=ROUTER_KINDS)
    p.add_argument("--n_layers", type=int, default=0)
    p.add_argument("--d_model", type=int, default=0)
    p.add_argument("--n_experts", type=int, default=0)
    p.add_argument("--vocab_size", type=int, default=0)
    p.add_argument("--max_new_tokens", type=int, default=32)
    p.add_argument("--out_json", default="weights/router_ablation.json")
    p.add_argument("--device", default=dev)
    p.set_defaults(fn=_cmd_router_ablate)

    p = sub.add_parser("env-audit", help="environment variables read, drift and unknown ones")
    p.add_argument("--root", default="", help="source root to scan (default: this package)")
    p.add_argument("--env_example", default="")
    p.add_argument("--prefix", default="OMNICODER_")
    p.add_argument("--out_json", default="weights/env_registry.json")
    p.add_argument("--out_index", default="")
    p.add_argument("--sync_example", action="store_true", help="append undocumented keys to --env_example")
    p.add_argument("--fail_on_drift", action="store_true")
    p.set_defaults(fn=_cmd_env_audit)

    p = sub.add_parser("gen-predictions", help="add predictions to a VQA / caption JSONL")
    p.add_argument("--task", default="vqa", choices=["vqa", "captions"])
    p.add_argument("--input", required=True)
    p.add_argument("--out", default="weights/predictions.jsonl")
    p.add_argument("--ckpt", default="", help="vision-language checkpoint (model, composer, config)")
    p.add_argument("--preset", default="tiny_moe")
    p.add_argument("--vision", default="vit_tiny")
    p.add_argument("--image_size", type=int, default=64)
    p.add_argument("--max_new_tokens", type=int, default=16)
    p.add_argument("--limit", type=int, default=0)
    p.add_argument("--device", default=dev)
    p.set_defaults(fn=_cmd_gen_predictions)

    p = sub.add_parser("latent-refine", help="refine continuous latents saved as .npy")
    p.add_argument("--latents", required=True)
    p.add_argument("--out_latents", required=True)
    p.add_argument("--ckpt", default="", help="refiner state_dict (or a dict with a 'refiner' entry)")
    p.add_argument("--hidden_mult", type=int, default=2)
    p.add_argument("--temporal", action="store_true")
    p.set_defaults(fn=_cmd_latent_refine)

    p = sub.add_parser("act-calibrate", help="activation maxima of the GEMM inputs and static int8 scales")
    p.add_argument("--preset", default="tiny_moe")
    p.add_argument("--ckpt", default="")
    p.add_argument("--prompts", nargs="*", default=None)
    p.add_argument("--max_tokens", type=int, default=256)
    p.add_argument("--decode_steps", type=int, default=8)
    p.add_argument("--out", default="weights/act_scales.json")
    p.add_argument("--device", default="cpu")
    p.set_defaults(fn=_cmd_act_calibrate)

    p = sub.add_parser("act-validate", help="check a calibration file or print a policy's knobs")
    p.add_argument("--policy", required=True)
    p.add_argument("--layers", type=int, default=0)
    p.set_defaults(fn=_cmd_act_validate)

    p = sub.add_parser("kv-dump", help="KV-cache rows of sample prompts, one .pt per prompt")
    p.add_argument("--preset", default="tiny_moe")
    p.add_argument("--ckpt", default="")
    p.add_argument("--prompts", nargs="*", default=None)
    p.add_argument("--max_tokens", type=int, default=512)
    p.add_argument("--out_dir", default="weights/kv_dump")
    p.add_argument("--device", default="cpu")
    p.set_defaults(fn=_cmd_kv_dump)

    p = sub.add_parser("kv-autoencoder", help="linear autoencoder of dumped KV rows")
    p.add_argument("--kv_dir", default="weights/kv_dump")
    p.add_argument("--latent", type=int, default=64)
    p.add_argument("--method", default="pca", choices=["pca", "sgd"])
    p.add_argument("--steps", type=int, default=500)
    p.add_argument("--lr", type=float, default=1e-3)
    p.add_argument("--out_pt", default="weights/kv_autoencoder.pt")
    p.add_argument("--out_json", default="weights/kv_compress_sidecar.json")
    p.set_defaults(fn=_cmd_kv_autoencoder)

    p = sub.add_parser("kv-prefetch", help="write the KV prefetch (pages kept) sidecar")
    p.add_argument("--out", default="weights/kv_prefetch.json")
    p.add_argument("--keep_pages", type=int, default=2)
    p.add_argument("--kv_paging_sidecar", default="")
    p.set_defaults(fn=_cmd_kv_prefetch)

    p = sub.add_parser("kv-retention", help="write the KV retention sidecar")
    p.add_argument("--out", required=True)
    p.add_argument("--compressive_slots", type=int, default=4)
    p.add_argument("--window_size", type=int, default=2048)
    p.set_defaults(fn=_cmd_kv_retention)

    p = sub.add_parser("code-verify", help="run a solution against a pytest file in the sandbox")
    p.add_argument("--code_file", default="")
    p.add_argument("--code_text", default="")
    p.add_argument("--tests_file", required=True)
    p.add_argument("--timeout", type=int, default=30)
    p.add_argument("--out_json", default="weights/code_verify_result.json")
    p.set_defaults(fn=_cmd_code_verify)

    p = sub.add_parser("auto-tune", help="speculative draft length from a measured acceptance benchmark")
    p.add_argument("--acceptance_json", default="weights/draft_acceptance.json")
    p.add_argument("--max_draft_len", type=int, default=16)
    p.add_argument("--out", default="weights/auto_tune.json")
    p.set_defaults(fn=_cmd_auto_tune)

    p = sub.add_parser("plot-metrics", help="SVG chart of a metrics JSON or of a JSONL training log")
    p.add_argument("--bench_json", default="")
    p.add_argument("--log_jsonl", default="")
    p.add_argument("--keys", default="", help="log: comma-separated keys to plot; JSON: substrings to keep")
    p.add_argument("--x", default="step", help="log: the x key (default: the row index when absent)")
    p.add_argument("--title", default="")
    p.add_argument("--out_svg", default="weights/metrics.svg")
    p.set_defaults(fn=_cmd_plot_metrics)

    p = sub.add_parser("write-threshold", help="write-policy acceptance threshold from teacher marks")
    p.add_argument("--marks", required=True, help="JSONL rows {text, write, optional score}")
    p.add_argument("--preset", default="tiny_moe")
    p.add_argument("--out", default="weights/write_policy_thresholds.json")
    p.set_defaults(fn=_cmd_write_threshold)
    return ap


def main(argv=None) -> int:
    a = _parser().parse_args(argv)
    return int(a.fn(a) or 0)


if __name__ == "__main__":
    sys.exit(main())
