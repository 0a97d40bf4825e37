"""Expert-parallel launcher: ``python -m omnicoder.tools.torchrun_ep --script
omnicoder.training.pretrain --devices cuda:0,cuda:1 [-- script args]``.

Starts one process per listed device with torch.distributed.run (rendezvous on
127.0.0.1, NCCL), restricting each job to the listed GPUs; the script then
trains expert parallel x data parallel over all ranks.  Inside an existing
torchrun job (RANK set) it runs the script in this process.

The reference launcher (src/omnicoder/tools/torchrun_ep.py:7-50) initialises a
process group in a single process, exports an environment variable that the
MoE layer in use never reads and runs the script unchanged: no rank ever holds
a subset of the experts.
"""
from __future__ import annotations

import argparse
import os
import runpy
import socket
import subprocess
import sys


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def build_command(script: str, devices: list[str], script_args: list[str], port: int | None = None,
                  max_restarts: int = 0) -> tuple[list[str], dict]:
    n = max(1, len(devices))
    env = dict(os.environ)
    ids = [d.split(":", 1)[1] for d in devices if d.startswith("cuda:")]
    if ids:
        env["CUDA_VISIBLE_DEVICES"] = ",".join(ids)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={port or _free_port()}", f"--max-restarts={max_restarts}",
           "-m", script] + script_args
    return cmd, env


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--script", default="omnicoder.training.pretrain")
    ap.add_argument("--devices", default="cuda:0")
    ap.add_argument("--max_restarts", type=int, default=0, help="elastic restarts of failed workers (torchrun)")
    ap.add_argument("--timeout", type=float, default=0, help="kill the whole job after this many seconds (0: none)")
    ap.add_argument("--dry_run", action="store_true")
    a, rest = ap.parse_known_args(argv)
    if rest and rest[0] == "--":
        rest = rest[1:]
    if "RANK" in os.environ and "WORLD_SIZE" in os.environ:
        sys.argv = [a.script] + rest
        runpy.run_module(a.script, run_name="__main__")
        return 0
    devices = [d.strip() for d in a.devices.split(",") if d.strip()]
    cmd, env = build_command(a.script, devices, rest, max_restarts=a.max_restarts)
    if a.dry_run:
        print(" ".join(cmd))
        return 0
    try:
        return subprocess.run(cmd, env=env, timeout=a.timeout or None).returncode
    except subprocess.TimeoutExpired:
        print(f"[torchrun_ep] job exceeded {a.timeout}s and was stopped", file=sys.stderr)
        return 124


if __name__ == "__main__":
    sys.exit(main())
