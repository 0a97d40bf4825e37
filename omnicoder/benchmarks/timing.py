"""Device timing helpers: CUDA events on the launching stream, L2 flush between
iterations, median over repetitions."""
from __future__ import annotations

import statistics

import torch

_FLUSH = None


def flush_l2():
    """Overwrite a 256 MiB buffer (the B200 L2 is 126 MB) so the next kernel starts cold."""
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    _FLUSH.fill_(1)


def time_fn(fn, iters: int = 10, warmup: int = 3, flush: bool = True) -> float:
    """Median milliseconds of `fn()` measured with CUDA events, L2 flushed before each run."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(iters):
        if flush:
            flush_l2()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return statistics.median(times)
