"""Performance counters and tracing (reference src/omnicoder/utils/perf.py:24-203).

* `add(name, seconds)` / `timer(name)` accumulate wall time per name (thread
  safe); `timer(name, cuda=True)` measures device time with CUDA events on the
  current stream instead; `snapshot()` returns {name: {count, total_s, mean_ms}}.
* `nvtx(name)` brackets a region with an NVTX range (visible in Nsight / ncu
  range filters); free when no profiler is attached.
* `enable_call_trace(path)` installs a sys.settrace call tracer that appends
  "call module:function" lines to a file (OMNICODER_TRACE_ALL=1 at import of
  omnicoder.utils.perf does the same); `disable_call_trace()` removes it.
* With OMNICODER_TIMING=1 the snapshot is written to
  $OMNICODER_LOG_DIR/perf_snapshot.json at interpreter exit.
"""
from __future__ import annotations

import atexit
import contextlib
import json
import os
import sys
import threading
import time

import torch

_lock = threading.Lock()
_stats: dict[str, list] = {}
_pending: list = []


def add(name: str, seconds: float) -> None:
    with _lock:
        s = _stats.setdefault(name, [0, 0.0])
        s[0] += 1
        s[1] += float(seconds)


@contextlib.contextmanager
def timer(name: str, cuda: bool = False):
    if cuda and torch.cuda.is_available():
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        try:
            yield
        finally:
            b.record()
            _pending.append((name, a, b))
    else:
        t0 = time.perf_counter()
        try:
            yield
        finally:
            add(name, time.perf_counter() - t0)


def _drain():
    while _pending:
        name, a, b = _pending.pop(0)
        b.synchronize()
        add(name, a.elapsed_time(b) / 1000.0)


def snapshot(reset_after: bool = False) -> dict:
    _drain()
    with _lock:
        out = {k: {"count": c, "total_s": t, "mean_ms": 1000.0 * t / max(1, c)} for k, (c, t) in _stats.items()}
        if reset_after:
            _stats.clear()
    return out


def reset() -> None:
    with _lock:
        _stats.clear()
    _pending.clear()


@contextlib.contextmanager
def nvtx(name: str):
    if torch.cuda.is_available():
        torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            torch.cuda.nvtx.range_pop()
    else:
        yield


_trace_file = None


def enable_call_trace(path: str) -> None:
    global _trace_file
    _trace_file = open(path, "a", buffering=1)

    def tracer(frame, event, arg):
        if event == "call":
            _trace_file.write(f"call {frame.f_globals.get('__name__', '?')}:{frame.f_code.co_name}\n")
        return None
    sys.settrace(tracer)
    threading.settrace(tracer)


def disable_call_trace() -> None:
    global _trace_file
    sys.settrace(None)
    threading.settrace(None)
    if _trace_file is not None:
        _trace_file.close()
        _trace_file = None


def _dump_at_exit():
    d = os.environ.get("OMNICODER_LOG_DIR", ".")
    try:
        with open(os.path.join(d, "perf_snapshot.json"), "w") as f:
            json.dump(snapshot(), f, indent=1)
    except Exception:
        pass


if os.environ.get("OMNICODER_TIMING") == "1":
    atexit.register(_dump_at_exit)
if os.environ.get("OMNICODER_TRACE_ALL") == "1":
    enable_call_trace(os.path.join(os.environ.get("OMNICODER_LOG_DIR", "."), "call_trace.log"))
