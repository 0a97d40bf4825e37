"""GGUF export of omnicoder models (and a reader for round trips).

The reference only shells out to llama.cpp's converter for Hugging Face LLaMA
checkpoints (src/omnicoder/export/gguf_export.py:1-122) and cannot write its
own models.  This writes any state_dict directly, following the public GGUF v3
layout: magic "GGUF", version, tensor count, metadata count, metadata
key/value pairs, tensor infos (name, dims innermost-first, type, offset), then
tensor data aligned to `general.alignment` (32).  Tensors are stored as F32,
F16 or BF16 (GGML type ids 0, 1, 30); the model config goes into
`omnicoder.config` as a JSON string and the architecture name into
`general.architecture`.
"""
from __future__ import annotations

import json
import struct

import numpy as np
import torch

GGUF_MAGIC = b"GGUF"
GGUF_VERSION = 3
ALIGN = 32
T_UINT32, T_INT32, T_FLOAT32, T_BOOL, T_STRING, T_UINT64, T_INT64 = 4, 5, 6, 7, 8, 10, 11
GGML_F32, GGML_F16, GGML_BF16 = 0, 1, 30
_DT = {GGML_F32: (torch.float32, 4), GGML_F16: (torch.float16, 2), GGML_BF16: (torch.bfloat16, 2)}


def _s(b: str) -> bytes:
    e = b.encode("utf-8")
    return struct.pack("<Q", len(e)) + e


def _kv(key: str, val) -> bytes:
    if isinstance(val, bool):
        return _s(key) + struct.pack("<I?", T_BOOL, val)
    if isinstance(val, int):
        if 0 <= val < 2 ** 32:
            return _s(key) + struct.pack("<II", T_UINT32, val)
        return _s(key) + (struct.pack("<IQ", T_UINT64, val) if val >= 0 else struct.pack("<Iq", T_INT64, val))
    if isinstance(val, float):
        return _s(key) + struct.pack("<If", T_FLOAT32, val)
    return _s(key) + struct.pack("<I", T_STRING) + _s(str(val))


def write_gguf(path: str, state_dict: dict, metadata: dict | None = None, dtype: str = "f16") -> None:
    ttype = {"f32": GGML_F32, "f16": GGML_F16, "bf16": GGML_BF16}[dtype]
    meta = {"general.alignment": ALIGN, **(metadata or {})}
    items = [(k, v.detach().cpu()) for k, v in state_dict.items() if torch.is_tensor(v) and v.is_floating_point()]
    infos, blobs, off = b"", [], 0
    for name, t in items:
        tt = GGML_F32 if t.dim() <= 1 else ttype                     # norms / biases stay f32
        data = t.to(_DT[tt][0]).contiguous()
        raw = data.view(torch.uint8).numpy().tobytes() if tt == GGML_BF16 else data.numpy().tobytes()
        dims = list(t.shape)[::-1] or [1]
        infos += _s(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        infos += struct.pack("<IQ", tt, off)
        pad = (-len(raw)) % ALIGN
        blobs.append(raw + b"\0" * pad)
        off += len(raw) + pad
    head = GGUF_MAGIC + struct.pack("<IQQ", GGUF_VERSION, len(items), len(meta))
    head += b"".join(_kv(k, v) for k, v in meta.items()) + infos
    head += b"\0" * ((-len(head)) % ALIGN)
    with open(path, "wb") as f:
        f.write(head)
        for b in blobs:
            f.write(b)


def read_gguf(path: str) -> tuple[dict, dict]:
    """Returns (metadata, {name: tensor}) for files written by write_gguf."""
    with open(path, "rb") as f:
        buf = f.read()
    assert buf[:4] == GGUF_MAGIC, "not a GGUF file"
    ver, nt, nkv = struct.unpack_from("<IQQ", buf, 4)
    p = 24

    def rs():
        nonlocal p
        (n,) = struct.unpack_from("<Q", buf, p)
        s = buf[p + 8:p + 8 + n].decode("utf-8")
        p += 8 + n
        return s

    meta = {}
    for _ in range(nkv):
        k = rs()
        (t,) = struct.unpack_from("<I", buf, p)
        p += 4
        if t == T_STRING:
            meta[k] = rs()
        elif t == T_UINT32:
            meta[k] = struct.unpack_from("<I", buf, p)[0]; p += 4
        elif t == T_UINT64:
            meta[k] = struct.unpack_from("<Q", buf, p)[0]; p += 8
        elif t == T_INT64:
            meta[k] = struct.unpack_from("<q", buf, p)[0]; p += 8
        elif t == T_FLOAT32:
            meta[k] = struct.unpack_from("<f", buf, p)[0]; p += 4
        elif t == T_BOOL:
            meta[k] = struct.unpack_from("<?", buf, p)[0]; p += 1
        else:
            raise ValueError(f"unsupported metadata type {t}")
    infos = []
    for _ in range(nt):
        name = rs()
        (nd,) = struct.unpack_from("<I", buf, p)
        dims = struct.unpack_from(f"<{nd}Q", buf, p + 4)
        tt, off = struct.unpack_from("<IQ", buf, p + 4 + 8 * nd)
        p += 4 + 8 * nd + 12
        infos.append((name, dims, tt, off))
    base = p + ((-p) % int(meta.get("general.alignment", ALIGN)))
    out = {}
    for name, dims, tt, off in infos:
        dt, es = _DT[tt]
        n = int(np.prod(dims))
        raw = buf[base + off: base + off + n * es]
        t = torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(dt) if tt == GGML_BF16 else \
            torch.from_numpy(np.frombuffer(raw, dtype={GGML_F32: np.float32, GGML_F16: np.float16}[tt]).copy())
        out[name] = t.reshape(list(dims)[::-1])
    return meta, out


def export_model_gguf(model, path: str, dtype: str = "f16") -> None:
    sd = model.export_state_dict() if hasattr(model, "export_state_dict") else model.state_dict()
    meta = {"general.architecture": "omnicoder", "general.name": getattr(getattr(model, "cfg", None), "name", "model")}
    if hasattr(model, "cfg"):
        meta["omnicoder.config"] = json.dumps(model.cfg.to_dict())
    write_gguf(path, sd, meta, dtype)
