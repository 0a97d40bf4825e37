"""HTTP serving: ``python -m omnicoder.tools.http_server --preset tiny_moe [--ckpt ...]``.

Endpoints (reference src/omnicoder/tools/http_server.py:147-1339):
  GET  /health                -> {"status": "ok", model info}
  POST /generate/text         {"prompt", "max_new_tokens", "temperature", "top_k", "top_p", "seed",
                               "repetition_penalty", "presence_penalty", "frequency_penalty"}
  POST /generate/unified      {"modality": "text", ...} (text only -> 501 for other modalities)
  POST /generate/image|video  {"prompt", "grid_h", "grid_w", "frames", "temperature", "top_k", "seed"}
                              -> {"shape", "layout", "pixels_b64"}: the model samples image / video
                              code tokens of the unified vocabulary and a VQ-VAE decoder renders
                              them (the reference calls external diffusion pipelines instead);
                              501 when the app was built without decoders

Unlike the reference (one request at a time per process), concurrent requests
are batched: a collector task takes up to `max_batch` queued requests that
share a prompt length and sampling settings and runs them as one batched
prefill + KV-cache decode.
"""
from __future__ import annotations

import argparse
import asyncio
import time

import torch

from ..inference.generate import generate
from ..training.tokenizer import get_tokenizer


_REQ = None


def _request_model():
    """The request body model, built on first use (pydantic is only needed for serving)."""
    global _REQ
    if _REQ is None:
        from pydantic import Field, create_model
        # out-of-range sampling settings are refused with 422 before they reach the sampler
        # (a repetition penalty <= 0 would divide logits by zero or flip their order)
        _REQ = (create_model("TextReq", prompt=(str, ...), max_new_tokens=(int, Field(64, ge=1)),
                             temperature=(float, 0.0), top_k=(int, Field(0, ge=0)),
                             top_p=(float, Field(1.0, gt=0.0, le=1.0)), seed=(int | None, None),
                             modality=(str, "text"), repetition_penalty=(float, Field(1.0, gt=0.0)),
                             presence_penalty=(float, 0.0), frequency_penalty=(float, 0.0)),
                create_model("MediaReq", prompt=(str, ...), grid_h=(int, 8), grid_w=(int, 8), frames=(int, 4),
                             temperature=(float, 1.0), top_k=(int, 0), seed=(int | None, None)))
    return _REQ


_UI_HTML = """<!doctype html><html><head><meta charset="utf-8"><title>omnicoder</title></head>
<body style="font-family:sans-serif;max-width:48em;margin:2em auto">
<h3>omnicoder</h3>
<textarea id="p" rows="6" style="width:100%">def fibonacci(n):</textarea><br>
max new tokens <input id="n" type="number" value="64"> temperature <input id="t" type="number" step="0.1" value="0.8">
<button onclick="go()">generate</button>
<pre id="o" style="white-space:pre-wrap;background:#f4f4f4;padding:1em"></pre>
<script>
async function go() {
  const body = {prompt: document.getElementById('p').value, max_new_tokens: +document.getElementById('n').value,
                temperature: +document.getElementById('t').value};
  const r = await fetch('/generate/text', {method: 'POST', headers: {'Content-Type': 'application/json'},
                                           body: JSON.stringify(body)});
  const j = await r.json();
  document.getElementById('o').textContent = j.text !== undefined ? j.text : JSON.stringify(j);
}
</script></body></html>"""


def create_app(model, tokenizer=None, max_batch: int = 16, batch_window_s: float = 0.005, image_vq=None,
               video_vq=None, vocab=None):
    """`image_vq` / `video_vq` (VQ-VAE decoders) and `vocab` (the unified vocabulary layout) enable
    /generate/image and /generate/video: the model samples code tokens of that modality and the
    decoder renders them; the response carries uint8 pixels (base64) and their shape."""
    from fastapi import FastAPI, HTTPException
    TextReq, MediaReq = _request_model()

    tok = tokenizer or get_tokenizer(model.cfg.vocab_size)
    dev = next(model.parameters()).device
    app = FastAPI(title="omnicoder")
    state = {"queue": None, "served": 0, "batches": 0}

    async def collector():
        q = state["queue"]
        while True:
            first = await q.get()
            group = [first]
            t_end = time.monotonic() + batch_window_s
            while len(group) < max_batch:
                timeout = t_end - time.monotonic()
                if timeout <= 0:
                    break
                try:
                    group.append(await asyncio.wait_for(q.get(), timeout))
                except asyncio.TimeoutError:
                    break
            buckets: dict = {}
            for item in group:
                r, ids, fut = item
                key = (ids.shape[1], r.max_new_tokens, r.temperature, r.top_k, r.top_p, r.seed,
                       r.repetition_penalty, r.presence_penalty, r.frequency_penalty)
                buckets.setdefault(key, []).append(item)
            for key, items in buckets.items():
                r0 = items[0][0]
                ids = torch.cat([it[1] for it in items]).to(dev)
                try:
                    out = await asyncio.to_thread(generate, model, ids, r0.max_new_tokens, r0.temperature, r0.top_k,
                                                  r0.top_p, seed=r0.seed, repetition_penalty=r0.repetition_penalty,
                                                  presence_penalty=r0.presence_penalty,
                                                  frequency_penalty=r0.frequency_penalty)
                    state["batches"] += 1
                    for i, (_, pid, fut) in enumerate(items):
                        fut.set_result(tok.decode(out[i, pid.shape[1]:].tolist()))
                except Exception as e:  # report to every waiting request
                    for _, _, fut in items:
                        if not fut.done():
                            fut.set_exception(e)

    @app.on_event("startup")
    async def _start():
        state["queue"] = asyncio.Queue()
        state["task"] = asyncio.create_task(collector())

    @app.get("/health")
    async def health():
        return {"status": "ok", "model": model.cfg.name, "device": str(dev), "served": state["served"],
                "batches": state["batches"]}

    @app.get("/")
    async def index():
        return {"service": "omnicoder", "model": model.cfg.name,
                "endpoints": ["GET /health", "GET /ui", "GET /metrics", "GET /debug/config", "POST /generate/text",
                              "POST /generate/unified", "POST /generate/image", "POST /generate/video"]}

    from fastapi.responses import HTMLResponse, PlainTextResponse

    @app.get("/ui", response_class=HTMLResponse)
    async def ui():
        return _UI_HTML

    @app.get("/metrics", response_class=PlainTextResponse)
    async def metrics():
        lines = ["# TYPE omnicoder_requests_served_total counter",
                 f"omnicoder_requests_served_total {state['served']}",
                 "# TYPE omnicoder_batches_total counter", f"omnicoder_batches_total {state['batches']}",
                 "# TYPE omnicoder_queue_depth gauge",
                 f"omnicoder_queue_depth {state['queue'].qsize() if state['queue'] is not None else 0}"]
        return "\n".join(lines) + "\n"

    @app.get("/debug/config")
    async def debug_config():
        return {"config": model.cfg.to_dict(), "max_batch": max_batch, "batch_window_s": batch_window_s,
                "image": image_vq is not None, "video": video_vq is not None}

    async def _text(r):
        ids = torch.tensor([tok.encode(r.prompt) or [0]])
        fut = asyncio.get_running_loop().create_future()
        await state["queue"].put((r, ids, fut))
        text = await fut
        state["served"] += 1
        return {"text": text, "prompt_tokens": int(ids.shape[1]), "new_tokens": r.max_new_tokens}

    async def gen_text(r):
        return await _text(r)

    async def gen_unified(r):
        if r.modality != "text":
            raise HTTPException(501, f"modality {r.modality!r} needs external generation weights")
        return await _text(r)

    gen_text.__annotations__ = {"r": TextReq}
    gen_unified.__annotations__ = {"r": TextReq}
    app.post("/generate/text")(gen_text)
    app.post("/generate/unified")(gen_unified)

    def _media(r, kind):
        import base64
        from ..multimodal.generation import generate_image, generate_video
        vq = image_vq if kind == "image" else video_vq
        if vq is None or vocab is None:
            raise HTTPException(501, f"{kind} generation needs a {kind} VQ decoder and the unified vocabulary "
                                     "layout (create_app(image_vq=..., video_vq=..., vocab=...))")
        ids = torch.tensor([tok.encode(r.prompt) or [0]], device=dev)
        gen = None
        if r.seed is not None:
            gen = torch.Generator(device=dev)
            gen.manual_seed(r.seed)
        kw = dict(grid=(r.grid_h, r.grid_w), temperature=r.temperature, top_k=r.top_k, generator=gen)
        out = (generate_image(model, vq, ids, vocab, **kw) if kind == "image"
               else generate_video(model, vq, ids, vocab, frames=r.frames, **kw))[0]
        pix = (out * 255).round().to(torch.uint8).cpu().contiguous()
        state["served"] += 1
        return {"shape": list(pix.shape), "layout": "CHW" if kind == "image" else "TCHW",
                "pixels_b64": base64.b64encode(pix.numpy().tobytes()).decode()}

    async def gen_image(r):
        return _media(r, "image")

    async def gen_video(r):
        return _media(r, "video")

    gen_image.__annotations__ = {"r": MediaReq}
    gen_video.__annotations__ = {"r": MediaReq}
    app.post("/generate/image")(gen_image)
    app.post("/generate/video")(gen_video)

    return app


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--ckpt", default=None)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8000)
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--max_batch", type=int, default=16)
    a = ap.parse_args(argv)
    from ..config import get_preset
    from ..inference.builders import load_model
    from ..models.lm import build_model
    model = load_model(a.ckpt, a.device, preset=a.preset)[0] if a.ckpt else build_model(get_preset(a.preset), a.device)
    import uvicorn
    uvicorn.run(create_app(model.eval(), max_batch=a.max_batch), host=a.host, port=a.port)


if __name__ == "__main__":
    main()
