"""Decode-step graph runners: generation through a session with onnxruntime's
interface, KV quantisation between steps, a simulated LRU page cache with
prefetch, and a decode-step throughput bench (reference
src/omnicoder/inference/runtimes/onnx_decode_generate.py:30-238,
kv_paging_runner.py:19-80, kv_prefetch.py:9-60, provider_bench.py:45-180).

A session is any object with `get_inputs()` / `get_outputs()` (items with
`.name` and `.shape`) and `run(output_names, feeds) -> list of arrays`:
  * `open_session(path)`: an onnxruntime InferenceSession over an exported
    decode-step graph (the export's I/O names: input_ids [, position],
    k_lat_i / v_lat_i -> logits, nk_lat_i / nv_lat_i);
  * `TorchStepSession(model)`: the same interface over the model's
    DecodeStepWrapper, so the runner works (and is tested) where onnxruntime
    is not installed, and serves as the oracle of an exported graph.
Compat-family graphs carry the fixed 16-slot latent window [B, H, 16, DL] per
layer; spec-family graphs carry a full cache [B, L, Hk, D] and a position input.
"""
from __future__ import annotations

import time
from collections import OrderedDict
from dataclasses import dataclass

import numpy as np
import torch


@dataclass
class TensorInfo:
    name: str
    shape: tuple


def providers() -> list[str]:
    """Execution providers onnxruntime offers here ([] when it is not installed)."""
    try:
        import onnxruntime as ort
    except ImportError:
        return []
    return list(ort.get_available_providers())


def open_session(path: str, provider_order: list[str] | None = None):
    try:
        import onnxruntime as ort
    except ImportError as e:
        raise RuntimeError("running an exported ONNX graph needs the `onnxruntime` package, which is not "
                           "installed; TorchStepSession runs the same decode step in PyTorch") from e
    avail = ort.get_available_providers()
    order = [p for p in (provider_order or ["CUDAExecutionProvider", "CPUExecutionProvider"]) if p in avail]
    return ort.InferenceSession(path, providers=order or avail)


class TorchStepSession:
    """onnxruntime-style session over DecodeStepWrapper(model)."""

    def __init__(self, model, max_len: int = 256, batch: int = 1):
        from ..export.onnx_export import DecodeStepWrapper, io_names
        self.step = DecodeStepWrapper(model).eval()
        L = len(model.blocks)
        ins, outs = io_names(L, spec=not self.step.compat)
        if self.step.compat:
            a = model.blocks[0].attn
            shape = (batch, a.n_heads, a.c.decode_window, a.dl)
        else:
            from ..export.onnx_export import spec_cache_shapes
            shape = spec_cache_shapes(model.cfg, batch, max_len)[0]     # MLA: the latent rows
        self._ins = [TensorInfo(n, (batch, 1) if n == "input_ids" else () if n == "position" else shape) for n in ins]
        self._outs = [TensorInfo(n, ()) for n in outs]
        self.device = next(model.parameters()).device

    def get_inputs(self):
        return list(self._ins)

    def get_outputs(self):
        return list(self._outs)

    @torch.no_grad()
    def run(self, output_names, feeds):
        args = [torch.as_tensor(np.asarray(feeds[i.name])).to(self.device) for i in self._ins]
        res = self.step(*args)
        named = {o.name: r for o, r in zip(self._outs, res)}
        return [named[n].float().cpu().numpy() for n in (output_names or [o.name for o in self._outs])]


def cache_layout(session):
    """(input token name, position name or None, [(k name, v name, shape)], output names)."""
    ins = session.get_inputs()
    names = [i.name for i in ins]
    ks = sorted((i for i in ins if i.name.startswith("k_lat_")), key=lambda i: int(i.name.rsplit("_", 1)[1]))
    vs = sorted((i for i in ins if i.name.startswith("v_lat_")), key=lambda i: int(i.name.rsplit("_", 1)[1]))
    if len(ks) != len(vs):
        raise RuntimeError("decode-step graph: mismatched k_lat / v_lat inputs")
    layers = [(k.name, v.name, tuple(k.shape)) for k, v in zip(ks, vs)]
    return names[0], ("position" if "position" in names else None), layers, [o.name for o in session.get_outputs()]


# ----------------------------------------------------------------------------
# Simulated KV page cache
# ----------------------------------------------------------------------------
@dataclass
class PagingConfig:
    n_layers: int
    page_len: int
    max_pages_ram: int
    prefetch_ahead: int = 1

    @classmethod
    def from_sidecars(cls, paging_json: str, prefetch_json: str | None = None,
                      prefetch_ahead: int = 1) -> "PagingConfig":
        """From the exporter's `.kv_paging.json` (page_len, n_layers) and a prefetch sidecar
        {"keep_pages": k}: k resident pages per layer (default 2)."""
        import json
        with open(paging_json) as f:
            pg = json.load(f)
        keep = 2
        if prefetch_json:
            with open(prefetch_json) as f:
                keep = max(1, int(json.load(f).get("keep_pages", keep)))
        L = int(pg["n_layers"])
        return cls(n_layers=L, page_len=int(pg["page_len"]), max_pages_ram=keep * L, prefetch_ahead=prefetch_ahead)


class LRUKVPager:
    """Pages keyed (layer, position // page_len) in an LRU of `max_pages_ram`
    entries.  Each decode position touches its page in every layer (a hit if
    resident, else a miss, counted as a stall unless an earlier prefetch brought
    it in) and prefetches the next `prefetch_ahead` pages of every layer."""

    def __init__(self, cfg: PagingConfig):
        self.cfg = cfg
        self.pages: OrderedDict = OrderedDict()          # key -> brought in by prefetch (not yet used)
        self.hits = self.misses = self.prefetches = self.prefetch_hits = self.stalls = 0

    def _insert(self, key, prefetched: bool) -> None:
        self.pages[key] = prefetched
        self.pages.move_to_end(key)
        while len(self.pages) > self.cfg.max_pages_ram:
            self.pages.popitem(last=False)

    def access(self, pos: int) -> None:
        page = pos // self.cfg.page_len
        for layer in range(self.cfg.n_layers):
            key = (layer, page)
            if key in self.pages:
                self.hits += 1
                if self.pages[key]:
                    self.prefetch_hits += 1
                self.pages[key] = False
                self.pages.move_to_end(key)
            else:
                self.misses += 1
                self.stalls += 1
                self._insert(key, False)
        for layer in range(self.cfg.n_layers):
            for a in range(1, self.cfg.prefetch_ahead + 1):
                key = (layer, page + a)
                if key not in self.pages:
                    self.prefetches += 1
                    self._insert(key, True)

    def stats(self) -> dict:
        total = max(1, self.hits + self.misses)
        return {"hits": self.hits, "misses": self.misses, "hit_rate": self.hits / total, "prefetches": self.prefetches,
                "prefetch_hits": self.prefetch_hits, "stalls": self.stalls, "resident_pages": len(self.pages)}


# ----------------------------------------------------------------------------
# Generation through a session
# ----------------------------------------------------------------------------
def _sample(logits: np.ndarray, temperature: float, top_k: int, top_p: float, rng: np.random.Generator) -> np.ndarray:
    """logits [B, V] -> ids [B]; greedy when temperature <= 0."""
    if temperature <= 0:
        return logits.argmax(-1)
    z = logits.astype(np.float64) / temperature
    if top_k > 0:
        kth = np.sort(z, -1)[:, -min(top_k, z.shape[-1])][:, None]
        z = np.where(z < kth, -np.inf, z)
    p = np.exp(z - z.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    if top_p < 1.0:
        order = np.argsort(-p, -1)
        sp = np.take_along_axis(p, order, -1)
        keep = np.cumsum(sp, -1) - sp < top_p
        mask = np.zeros_like(p, dtype=bool)
        np.put_along_axis(mask, order, keep, -1)
        p = np.where(mask, p, 0.0)
        p /= p.sum(-1, keepdims=True)
    return np.array([rng.choice(p.shape[-1], p=row) for row in p])


class DecodeRunner:
    """Token-by-token generation through a decode-step session.  kv_quant "u8" /
    "nf4" stores the cache between steps in that format (grouped along the last
    dim, `group` wide) and dequantises it for the next feed; `pager` records the
    page accesses of every position."""

    def __init__(self, session, kv_quant: str | None = None, group: int = 64, pager: LRUKVPager | None = None,
                 logit_bias: dict[int, float] | None = None, bias_alpha: float = 1.0):
        self.session = session
        self.tok_name, self.pos_name, self.layers, self.out_names = cache_layout(session)
        self.kv_quant, self.group, self.pager = kv_quant, group, pager
        self.logit_bias, self.bias_alpha = logit_bias or {}, bias_alpha

    @classmethod
    def from_sidecars(cls, session, model_path: str, prefetch_json: str | None = None, **kw) -> "DecodeRunner":
        """A runner configured by the sidecars the exporter wrote beside `model_path`: `.kvq.json`
        (cache format and group) and `.kv_paging.json` (+ an optional prefetch sidecar) for the pager."""
        import json
        import os
        base = model_path[:-5] if model_path.endswith(".onnx") else model_path
        kvq, group, pager = None, 64, None
        if os.path.exists(base + ".kvq.json"):
            with open(base + ".kvq.json") as f:
                meta = json.load(f)
            kvq, group = meta["scheme"], int(meta.get("group", 64))
        if os.path.exists(base + ".kv_paging.json"):
            pager = LRUKVPager(PagingConfig.from_sidecars(base + ".kv_paging.json", prefetch_json))
        return cls(session, kv_quant=kvq, group=group, pager=pager, **kw)

    def _zeros(self, batch: int) -> list[np.ndarray]:
        out = []
        for _, _, shape in self.layers:
            out += [np.zeros((batch,) + tuple(int(s) for s in shape[1:]), np.float32)] * 2
        return out

    def _store(self, cache: list[np.ndarray]):
        if not self.kv_quant:
            return cache
        from ..quant.kv import quantize_kv
        return [quantize_kv(torch.from_numpy(cache[i]), torch.from_numpy(cache[i + 1]), self.kv_quant, self.group)
                for i in range(0, len(cache), 2)]

    def _load(self, stored) -> list[np.ndarray]:
        if not self.kv_quant:
            return stored
        from ..quant.kv import dequantize_kv
        out = []
        for kq, vq, meta in stored:
            k, v = dequantize_kv(kq, vq, meta)
            out += [k.numpy(), v.numpy()]
        return out

    def step(self, tokens: np.ndarray, pos: int, cache: list[np.ndarray]):
        feeds = {self.tok_name: tokens.astype(np.int64).reshape(-1, 1)}
        if self.pos_name:
            feeds[self.pos_name] = np.array(pos, dtype=np.int64)
        for (kn, vn, _), i in zip(self.layers, range(0, len(cache), 2)):
            feeds[kn], feeds[vn] = cache[i], cache[i + 1]
        res = self.session.run(self.out_names, feeds)
        logits = np.asarray(res[0]).reshape(tokens.shape[0], -1)
        for t, b in self.logit_bias.items():
            logits[:, t] += self.bias_alpha * b
        if self.pager is not None:
            self.pager.access(pos)
        return logits, [np.asarray(r, np.float32) for r in res[1:]]

    def generate(self, prompt: np.ndarray, max_new_tokens: int, temperature: float = 0.0, top_k: int = 0,
                 top_p: float = 1.0, seed: int = 0, eos_id: int | None = None) -> np.ndarray:
        """prompt [B, S] int -> [B, S + n] (prompt fed one token per step, as the graph takes one)."""
        rng = np.random.default_rng(seed)
        B, S = prompt.shape
        stored = self._store(self._zeros(B))
        ids = [prompt[:, i] for i in range(S)]
        logits = None
        for pos in range(S):
            logits, cache = self.step(prompt[:, pos], pos, self._load(stored))
            stored = self._store(cache)
        for n in range(max_new_tokens):
            nxt = _sample(logits, temperature, top_k, top_p, rng)
            ids.append(nxt)
            if eos_id is not None and bool((nxt == eos_id).all()):
                break
            if n + 1 < max_new_tokens:
                logits, cache = self.step(nxt, S + n, self._load(stored))
                stored = self._store(cache)
        return np.stack(ids, 1)


def bench_decode(session, vocab_size: int, prompt_len: int = 16, gen_tokens: int = 32, seed: int = 0) -> float:
    """Decode-step throughput (tokens/s) of a session after feeding a random prompt."""
    rng = np.random.default_rng(seed)
    runner = DecodeRunner(session)
    cache = runner._zeros(1)
    for pos in range(prompt_len):
        _, cache = runner.step(rng.integers(0, vocab_size, (1,)), pos, cache)
    t0 = time.perf_counter()
    for i in range(gen_tokens):
        _, cache = runner.step(rng.integers(0, vocab_size, (1,)), prompt_len + i, cache)
    return gen_tokens / max(time.perf_counter() - t0, 1e-9)
