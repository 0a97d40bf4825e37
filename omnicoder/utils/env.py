"""Environment variables (reference src/omnicoder/utils/env_registry.py:11-185,
env_defaults.py, inference/gen_config.py).

This framework reads configuration from typed dataclasses and CLI flags; the
environment is only used for launcher plumbing and logging.  The registry
scans the package source for the environment variables it reads so the set is
documented, `load_dotenv` applies a KEY=VALUE file without overriding what is
already set, and `runtime_snapshot` freezes the relevant variables once (so
hot loops never call os.getenv).
"""
from __future__ import annotations

import os
import re

_PATTERN = re.compile(r"""(?:os\.environ\.get|os\.getenv|os\.environ\[)\(?\s*["']([A-Z][A-Z0-9_]+)["']""")


def scan_registry(root: str | None = None) -> dict[str, list[str]]:
    """{VARIABLE: [file:line, ...]} for every environment read under `root` (default: this package)."""
    root = root or os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out: dict[str, list[str]] = {}
    for d, _, files in os.walk(root):
        for f in files:
            if not f.endswith(".py"):
                continue
            p = os.path.join(d, f)
            with open(p, encoding="utf-8", errors="replace") as fh:
                for i, line in enumerate(fh, 1):
                    for m in _PATTERN.finditer(line):
                        out.setdefault(m.group(1), []).append(f"{os.path.relpath(p, root)}:{i}")
    return dict(sorted(out.items()))


def registry_markdown(reg: dict[str, list[str]]) -> str:
    lines = ["| variable | read at |", "|---|---|"]
    lines += [f"| `{k}` | {', '.join(v)} |" for k, v in reg.items()]
    return "\n".join(lines)


def load_dotenv(path: str = ".env", override: bool = False) -> dict[str, str]:
    applied = {}
    if not os.path.exists(path):
        return applied
    with open(path) as f:
        for line in f:
            line = line.strip()
            if not line or line.startswith("#") or "=" not in line:
                continue
            k, v = line.split("=", 1)
            k, v = k.strip(), v.strip().strip('"').strip("'")
            if override or k not in os.environ:
                os.environ[k] = v
                applied[k] = v
    return applied


def runtime_snapshot(prefix: str = "OMNICODER_") -> dict[str, str]:
    return {k: v for k, v in os.environ.items() if k.startswith(prefix)}
