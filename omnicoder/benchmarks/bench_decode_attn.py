"""Decode attention microbenchmark: B sequences, one new token each (or Tn for
speculative verification), against an MLA latent cache (576 = 512 latent + 64
rope dims, value = latent) of `ctx` tokens, int8 or bf16, optional sliding
window and memory rows.

    python -m omnicoder.benchmarks.bench_decode_attn [--batch 64 --ctx 8192 --window 4096 --mem 64 --kv int8]

Reports the CUDA-event time of one call (median of `--iters`, the cache is
larger than L2 so every call streams it from HBM) and the achieved cache-read
bandwidth (bytes of the visible rows / time).
"""
from __future__ import annotations

import argparse
import json
import math

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--ctx", type=int, default=8192)
    ap.add_argument("--tn", type=int, default=1)
    ap.add_argument("--heads", type=int, default=16)
    ap.add_argument("--window", type=int, default=4096)
    ap.add_argument("--mem", type=int, default=64)
    ap.add_argument("--kv", default="int8", choices=["int8", "bf16"])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--mha", type=int, default=0, metavar="KV_HEADS",
                    help="MHA / GQA cache with this many kv heads (head dim --head-dim) instead of the MLA latent")
    ap.add_argument("--head-dim", type=int, default=128)
    a = ap.parse_args(argv)
    from omnicoder.inference.kv_cache import quantize_int8
    from omnicoder.ops import _ext
    from omnicoder.ops.decode import decode_attention
    dev = torch.device("cuda")
    B, Tn, H = a.batch, a.tn, a.heads
    DQ, DV = (a.head_dim, a.head_dim) if a.mha else (576, 512)
    L = a.mem + a.ctx + Tn
    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randn(B, Tn, H, DQ, generator=g).to(dev, torch.bfloat16)
    v = vs = ks = None
    if a.mha:
        k = torch.randn(B, L, a.mha, DQ, device=dev, dtype=torch.bfloat16)
        v = torch.randn(B, L, a.mha, DV, device=dev, dtype=torch.bfloat16)
    else:
        k = torch.randn(B, L, DQ, device=dev, dtype=torch.bfloat16)
    if a.kv == "int8":
        k, ks = quantize_int8(k, -1)
        if v is not None:
            v, vs = quantize_int8(v, -1)
    kv_len = torch.full((B,), a.ctx + Tn, dtype=torch.int32, device=dev)
    q_pos = (kv_len[:, None] - Tn + torch.arange(Tn, device=dev)[None, :]).to(torch.int32)
    kw = dict(window=a.window, scale=1.0 / math.sqrt(DQ), k_scale=ks, v_scale=vs, latent_v_dim=0 if a.mha else DV,
              sink_rows=a.mem, n_sink=a.mem)
    for _ in range(3):
        decode_attention(q, k, v, q_pos, kv_len, **kw)
    torch.cuda.synchronize()
    times = []
    for _ in range(a.iters):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        decode_attention(q, k, v, q_pos, kv_len, **kw)
        e1.record()
        e1.synchronize()
        times.append(e0.elapsed_time(e1))
    _ext.check_status()
    times.sort()
    ms = times[len(times) // 2]
    rows = (min(a.ctx + Tn, a.window + Tn - 1) if a.window else a.ctx + Tn) + a.mem
    row_bytes = (a.mha * (DQ + DV) if a.mha else DQ) * (1 if a.kv == "int8" else 2)
    row_bytes += (4 * (2 * a.mha if a.mha else 1)) if a.kv == "int8" else 0
    nbytes = B * rows * row_bytes
    print(json.dumps({"kernel": f"decode attention ({'MHA/GQA %d kv heads x %d' % (a.mha, DQ) if a.mha else 'MLA latent'})", "batch": B, "tn": Tn, "heads": H, "ctx": a.ctx,
                      "window": a.window, "mem": a.mem, "kv": a.kv, "ms": ms,
                      "gbs": nbytes / ms / 1e6, "bytes": nbytes}))


if __name__ == "__main__":
    main()
