"""Failure detection between steps and host-side fault injection for
multi-process jobs.

The reference has no failure detection beyond subprocess timeouts, a data
loader retry and atomic saves (src/omnicoder/tools/run_training.py:106-125,
src/omnicoder/training/pretrain.py:243-250, src/omnicoder/utils/torchutils.py:302-345).

Heartbeat: every rank publishes "<beat>:<step>" under <prefix>/<rank> in the
job's c10d store, from a daemon thread every `interval` seconds (the beat
counter proves the process is alive) and from the training loop when it is
about to run a step.  `check(step)`, called by every rank before the step's
first launch, publishes `step` and returns once every other rank has published
a step >= `step`; it raises RankFailure naming the rank when one
  * announced that it left (`leave()`, e.g. on a caught exception),
  * never published within `timeout` of the check's start ("never joined"),
  * published no new beat for `timeout` seconds (process gone or frozen), or
  * kept beating but did not reach `step` within `stall_timeout` (main loop hung).
Liveness is judged by changes of the beat counter seen on this host's own
monotonic clock, so clocks of different hosts never enter.  No device work
is involved: a rank only leaves between steps, with no kernel or collective in
flight, and the others learn of it before their next launch.

FaultInjector makes the failures on the host, at a given rank and step:
"raise" (an exception in the training loop), "exit" (the process ends at once,
without cleanup), "hang" (the heartbeat stops and the loop sleeps), "stall"
(the loop sleeps while the heartbeat thread keeps beating) and "drop" (`drop()`
tells a transport to lose that step's message).  Spec syntax, also
read from OMNICODER_FAULT: "rank=1,step=3,kind=exit[,seconds=30]".
"""
from __future__ import annotations

import os
import threading
import time
from dataclasses import dataclass

import torch.distributed as dist


class RankFailure(RuntimeError):
    def __init__(self, rank: int, reason: str):
        super().__init__(f"rank {rank} failed: {reason}")
        self.rank, self.reason = rank, reason


class Heartbeat:
    def __init__(self, store=None, rank: int | None = None, world: int | None = None, interval: float = 0.2,
                 timeout: float = 5.0, stall_timeout: float | None = None, prefix: str = "omnicoder/hb"):
        self.store = store if store is not None else dist.distributed_c10d._get_default_store()
        self.rank = dist.get_rank() if rank is None else rank
        self.world = dist.get_world_size() if world is None else world
        self.interval, self.timeout = interval, timeout
        self.stall_timeout = stall_timeout if stall_timeout is not None else 4 * timeout
        self.prefix = prefix
        self._beat = 0
        self._step = -1
        self._lock = threading.Lock()
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        self._seen: dict[int, tuple[int, float]] = {}    # rank -> (last beat counter, local time it changed)

    # -- publishing ----------------------------------------------------------
    def _publish(self):
        with self._lock:
            self._beat += 1
            self.store.set(f"{self.prefix}/{self.rank}", f"{self._beat}:{self._step}")

    def _run(self):
        while not self._stop.wait(self.interval):
            self._publish()

    def start(self) -> "Heartbeat":
        self._publish()
        self._thread = threading.Thread(target=self._run, name="omnicoder-heartbeat", daemon=True)
        self._thread.start()
        return self

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=2 * self.interval + 1)
            self._thread = None

    def leave(self, reason: str = "left") -> bool:
        """Stop beating and announce the departure; False when the store no longer answers (the
        store host, rank 0, is gone), so a caller unwinding from an error keeps its own exception."""
        self.stop()
        try:
            self.store.set(f"{self.prefix}/left/{self.rank}", reason)
            return True
        except (RuntimeError, ConnectionError, OSError):
            return False

    # -- checking ------------------------------------------------------------
    def _read(self, r: int):
        key = f"{self.prefix}/{r}"
        if not self.store.check([key]):
            return None
        beat, step = self.store.get(key).decode().split(":")
        return int(beat), int(step)

    def check(self, step: int, ranks=None):
        """Announce that this rank is about to run `step` and block until every other rank has
        announced it too; raise RankFailure otherwise (rank 0 when the store, which rank 0
        hosts, stops answering)."""
        try:
            self._check(step, ranks)
        except RankFailure:
            raise
        except (RuntimeError, ConnectionError, OSError) as e:
            raise RankFailure(0, f"store unreachable ({e})") from e

    def _check(self, step: int, ranks):
        self._step = step
        self._publish()
        t0 = time.monotonic()
        pending = [r for r in (ranks if ranks is not None else range(self.world)) if r != self.rank]
        while pending:
            now = time.monotonic()
            for r in list(pending):
                if self.store.check([f"{self.prefix}/left/{r}"]):
                    raise RankFailure(r, self.store.get(f"{self.prefix}/left/{r}").decode())
                got = self._read(r)
                if got is None:
                    if now - t0 > self.timeout:
                        raise RankFailure(r, f"never joined within {self.timeout:.1f} s")
                    continue
                beat, rstep = got
                last = self._seen.get(r)
                if last is None or last[0] != beat:
                    self._seen[r] = (beat, now)
                elif now - last[1] > self.timeout:
                    raise RankFailure(r, f"no heartbeat for {now - last[1]:.1f} s")
                if rstep >= step:
                    pending.remove(r)
                elif now - t0 > self.stall_timeout:
                    raise RankFailure(r, f"stalled before step {rstep + 1} (waiting for step {step})")
            if pending:
                time.sleep(min(0.05, self.interval))


class StoreChannel:
    """Small control messages between ranks through the store: `send(dst, tag, text)`,
    `recv(src, tag)` waits at most `timeout` seconds and raises RankFailure(src) when the
    message never arrives (a lost message or a dead sender)."""

    def __init__(self, store=None, rank: int | None = None, timeout: float = 5.0, prefix: str = "omnicoder/msg"):
        self.store = store if store is not None else dist.distributed_c10d._get_default_store()
        self.rank = dist.get_rank() if rank is None else rank
        self.timeout, self.prefix = timeout, prefix

    def send(self, dst: int, tag: str, text: str):
        self.store.set(f"{self.prefix}/{self.rank}->{dst}/{tag}", text)

    def recv(self, src: int, tag: str) -> str:
        key = f"{self.prefix}/{src}->{self.rank}/{tag}"
        t0 = time.monotonic()
        while not self.store.check([key]):
            if time.monotonic() - t0 > self.timeout:
                raise RankFailure(src, f"message {tag!r} not received within {self.timeout:.1f} s")
            time.sleep(0.01)
        return self.store.get(key).decode()


# ----------------------------------------------------------------------------
# Host-side fault injection
# ----------------------------------------------------------------------------
class InjectedFault(RuntimeError):
    pass


@dataclass
class FaultSpec:
    rank: int
    step: int
    kind: str                 # raise | exit | hang | stall | drop
    seconds: float = 3600.0   # how long "hang" / "stall" sleep

    @classmethod
    def parse(cls, text: str) -> "FaultSpec":
        kv = dict(part.split("=", 1) for part in text.split(",") if part.strip())
        spec = cls(int(kv["rank"]), int(kv["step"]), kv["kind"], float(kv.get("seconds", 3600.0)))
        if spec.kind not in ("raise", "exit", "hang", "stall", "drop"):
            raise ValueError(f"unknown fault kind {spec.kind!r}")
        return spec


# kinds that end or freeze a rank's process without unwinding it; on GPU ranks of a
# multi-rank job they can leave peers waiting on device barriers or leave memory bound
# to an NVLink multicast object, so they are only armed on CPU (gloo) ranks
HOST_ONLY_KINDS = ("exit", "hang", "stall")


class FaultInjector:
    def __init__(self, specs=None):
        self.specs = list(specs or [])

    @classmethod
    def from_env(cls, var: str = "OMNICODER_FAULT", device_type: str = "cpu", world: int = 1) -> "FaultInjector":
        """Fault specs from `var` ("rank=1,step=3,kind=raise;..."). On a CUDA job with more
        than one rank only the unwinding kinds (raise, drop) are accepted: an exiting,
        hanging or stalled GPU rank may be holding peer-mapped (symmetric / multicast)
        memory or be awaited by peers' device barriers."""
        text = os.environ.get(var, "")
        inj = cls([FaultSpec.parse(t) for t in text.split(";") if t.strip()])
        inj.check_allowed(device_type, world)
        return inj

    def check_allowed(self, device_type: str, world: int):
        if device_type == "cuda" and world > 1:
            bad = [s.kind for s in self.specs if s.kind in HOST_ONLY_KINDS]
            if bad:
                raise ValueError(f"fault kinds {sorted(set(bad))} are only injected on CPU (gloo) ranks; "
                                 "on multi-rank CUDA jobs use kind=raise or kind=drop")

    def _match(self, rank: int, step: int, kinds) -> FaultSpec | None:
        for s in self.specs:
            if s.rank == rank and s.step == step and s.kind in kinds:
                return s
        return None

    def at_step(self, rank: int, step: int, heartbeat: Heartbeat | None = None):
        """Called by the training loop between steps (nothing in flight on the device)."""
        s = self._match(rank, step, ("raise", "exit", "hang", "stall"))
        if s is None:
            return
        if s.kind == "raise":
            raise InjectedFault(f"injected failure at rank {rank}, step {step}")
        if s.kind == "exit":
            os._exit(17)
        if s.kind == "hang" and heartbeat is not None:
            heartbeat.stop()
        time.sleep(s.seconds)

    def drop(self, rank: int, step: int) -> bool:
        return self._match(rank, step, ("drop",)) is not None
