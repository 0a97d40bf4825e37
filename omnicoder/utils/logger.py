"""Logging (reference src/omnicoder/utils/logger.py:17-141): `get_logger(name)`
returns a logger under the `omnicoder` hierarchy with a console handler and,
when OMNICODER_LOG_DIR (or `log_dir`) is set, a size-rotated file handler.
Handlers never raise into the caller (a failing sink is dropped)."""
from __future__ import annotations

import logging
import logging.handlers
import os
import sys

_CONFIGURED = False


class _SafeHandler(logging.Handler):
    def __init__(self, inner: logging.Handler):
        super().__init__(inner.level)
        self.inner = inner

    def emit(self, record):
        try:
            self.inner.emit(record)
        except Exception:
            pass

    def setFormatter(self, fmt):
        self.inner.setFormatter(fmt)


def configure(level: str | int | None = None, log_dir: str | None = None) -> logging.Logger:
    global _CONFIGURED
    root = logging.getLogger("omnicoder")
    if _CONFIGURED and level is None and log_dir is None:
        return root
    root.setLevel(level or os.environ.get("OMNICODER_LOG_LEVEL", "INFO"))
    root.handlers.clear()
    fmt = logging.Formatter("%(asctime)s %(levelname)s [%(name)s] %(message)s")
    h = _SafeHandler(logging.StreamHandler(sys.stderr))
    h.setFormatter(fmt)
    root.addHandler(h)
    d = log_dir or os.environ.get("OMNICODER_LOG_DIR")
    if d:
        os.makedirs(d, exist_ok=True)
        fh = _SafeHandler(logging.handlers.RotatingFileHandler(os.path.join(d, "omnicoder.log"), maxBytes=64 << 20,
                                                               backupCount=3))
        fh.setFormatter(fmt)
        root.addHandler(fh)
    root.propagate = False
    _CONFIGURED = True
    return root


def get_logger(name: str = "omnicoder") -> logging.Logger:
    configure()
    return logging.getLogger(name if name.startswith("omnicoder") else f"omnicoder.{name}")
