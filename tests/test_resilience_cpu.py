"""Failure detection and recovery on CPU ranks (gloo): every failure is made on the
host (a rank that raises, exits, hangs or stalls between steps; a dropped message;
a corrupted checkpoint), never on a device.  The surviving ranks must name the
failed rank within the time limit instead of blocking in a collective, and a
relaunched run must resume from the last good checkpoint and end with the same
weights as an uninterrupted run."""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _DPTrainer:
    """Minimal data-parallel trainer: gradient all_reduce + SGD on a linear layer."""

    def __init__(self):
        torch.manual_seed(0)
        self.model = nn.Linear(8, 4)
        self.step_idx = 0

    def step(self, ids, labels):
        loss = ((self.model(ids) - labels) ** 2).mean()
        loss.backward()
        for p in self.model.parameters():
            dist.all_reduce(p.grad)
            p.data.add_(p.grad, alpha=-0.01)
            p.grad = None
        self.step_idx += 1
        return type("S", (), {"loss": loss.detach()})()

    def state_dict(self):
        return {"step": self.step_idx}

    def load_state_dict(self, sd):
        self.step_idx = sd["step"]


def _batch(step):
    g = torch.Generator().manual_seed(step)
    return torch.randn(4, 8, generator=g), torch.randn(4, 4, generator=g)


def _worker(rank, world, port, fault, use_heartbeat, tmp, q, release):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=4))
    from omnicoder.parallel.health import FaultInjector, FaultSpec, Heartbeat, RankFailure
    from omnicoder.training.resilience import CheckpointManager, train_with_recovery
    hb = Heartbeat(interval=0.1, timeout=1.5, stall_timeout=3.0).start() if use_heartbeat else None
    inj = FaultInjector([FaultSpec.parse(fault)] if fault else [])
    t0 = time.monotonic()
    try:
        train_with_recovery(_DPTrainer(), _batch, 8, CheckpointManager(os.path.join(tmp, f"r{rank}"), rank=rank),
                            save_every=100, heartbeat=hb, injector=inj, rank=rank)
        q.put((rank, "done", None, time.monotonic() - t0))
    except RankFailure as e:
        q.put((rank, "rank_failure", (e.rank, e.reason), time.monotonic() - t0))
    except Exception as e:  # injected exception, or a collective that ended with an error
        q.put((rank, type(e).__name__, str(e)[:200], time.monotonic() - t0))
    q.close()
    q.join_thread()   # flush the result before leaving
    if rank == 0:     # rank 0 hosts the store: keep it up until every surviving rank has reported
        release.wait(timeout=30)
    os._exit(0)       # no destroy_process_group: peers may be gone


def _run(world, fault, use_heartbeat, tmp_path, expect_exit=()):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    release = ctx.Event()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fault, use_heartbeat, str(tmp_path), q, release))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(world - len(expect_exit)):
            rank, kind, info, secs = q.get(timeout=60)
            out[rank] = (kind, info, secs)
    finally:
        release.set()
        for p in procs:
            p.join(timeout=5)
            if p.is_alive():      # the hung / stalled rank: our own child process
                p.terminate()
                p.join(timeout=5)
    return out, procs


def test_exited_rank_is_named_by_heartbeat(tmp_path):
    out, procs = _run(3, "rank=2,step=3,kind=exit", True, tmp_path, expect_exit=(2,))
    assert procs[2].exitcode == 17
    for r in (0, 1):
        kind, info, secs = out[r]
        assert kind == "rank_failure" and info[0] == 2 and "heartbeat" in info[1], out
        assert secs < 20


def test_raising_rank_announces_leave(tmp_path):
    out, _ = _run(3, "rank=1,step=2,kind=raise", True, tmp_path)
    assert out[1][0] == "InjectedFault"
    for r in (0, 2):
        kind, info, _ = out[r]
        assert kind == "rank_failure" and info[0] == 1 and "InjectedFault" in info[1], out


def test_hung_rank_without_heartbeat_is_detected(tmp_path):
    out, _ = _run(2, "rank=1,step=2,kind=hang,seconds=60", True, tmp_path, expect_exit=(1,))
    kind, info, secs = out[0]
    assert kind == "rank_failure" and info[0] == 1 and "heartbeat" in info[1], out
    assert secs < 20


def test_stalled_rank_with_live_heartbeat_is_detected(tmp_path):
    out, _ = _run(2, "rank=1,step=1,kind=stall,seconds=60", True, tmp_path, expect_exit=(1,))
    kind, info, _ = out[0]
    assert kind == "rank_failure" and info[0] == 1 and "stalled" in info[1], out


def test_collective_timeout_without_heartbeat(tmp_path):
    """Without the heartbeat a dead peer ends the next collective with an error (short
    process-group timeout), not a hang."""
    out, _ = _run(2, "rank=1,step=2,kind=raise", False, tmp_path)
    assert out[1][0] == "InjectedFault"
    kind, _, secs = out[0]
    assert kind not in ("done", "rank_failure") and secs < 30, out


def _channel_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from omnicoder.parallel.health import FaultInjector, FaultSpec, RankFailure, StoreChannel
    ch = StoreChannel(timeout=1.0)
    inj = FaultInjector([FaultSpec.parse("rank=0,step=2,kind=drop")])
    got = []
    for step in range(4):
        if rank == 0:
            if not inj.drop(0, step):
                ch.send(1, f"s{step}", f"hello {step}")
        else:
            try:
                got.append(ch.recv(0, f"s{step}"))
            except RankFailure as e:
                got.append(f"lost from {e.rank}")
    q.put((rank, got))
    dist.barrier()
    dist.destroy_process_group()


def test_dropped_message_is_reported():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_channel_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=60) for _ in procs)
    for p in procs:
        p.join(timeout=30)
    assert res[1] == ["hello 0", "hello 1", "lost from 0", "hello 3"]


def test_fault_spec_parsing(monkeypatch):
    from omnicoder.parallel.health import FaultInjector, FaultSpec
    s = FaultSpec.parse("rank=3,step=7,kind=hang,seconds=2.5")
    assert (s.rank, s.step, s.kind, s.seconds) == (3, 7, "hang", 2.5)
    with pytest.raises(ValueError):
        FaultSpec.parse("rank=0,step=0,kind=segfault")
    monkeypatch.setenv("OMNICODER_FAULT_TEST", "rank=0,step=1,kind=drop;rank=1,step=2,kind=raise")
    inj = FaultInjector.from_env("OMNICODER_FAULT_TEST")
    assert inj.drop(0, 1) and not inj.drop(0, 2) and len(inj.specs) == 2


def test_fault_injector_refuses_process_ending_kinds_on_gpu_jobs(monkeypatch):
    """exit / hang / stall are armed only on CPU ranks; a multi-rank CUDA job accepts raise / drop."""
    from omnicoder.parallel.health import FaultInjector
    for kind in ("exit", "hang", "stall"):
        monkeypatch.setenv("OMNICODER_FAULT_TEST", f"rank=1,step=2,kind={kind}")
        with pytest.raises(ValueError):
            FaultInjector.from_env("OMNICODER_FAULT_TEST", device_type="cuda", world=2)
        assert len(FaultInjector.from_env("OMNICODER_FAULT_TEST", device_type="cpu", world=2).specs) == 1
        assert len(FaultInjector.from_env("OMNICODER_FAULT_TEST", device_type="cuda", world=1).specs) == 1
    monkeypatch.setenv("OMNICODER_FAULT_TEST", "rank=1,step=2,kind=raise;rank=0,step=1,kind=drop")
    assert len(FaultInjector.from_env("OMNICODER_FAULT_TEST", device_type="cuda", world=8).specs) == 2


def test_resume_from_last_good_checkpoint(tmp_path):
    """An injected failure at step 5 (checkpoints every 2 steps) and a corrupted newest
    checkpoint: the relaunch resumes from step 2 and ends equal to an uninterrupted run,
    optimiser moments included."""
    from omnicoder.config import MoEConfig, ModelConfig, TrainConfig, AttentionConfig
    from omnicoder.models.lm import build_model
    from omnicoder.parallel.health import FaultInjector, FaultSpec, InjectedFault
    from omnicoder.training.engine import Trainer, synthetic_batch
    from omnicoder.training.resilience import CheckpointManager, train_with_recovery

    cfg = ModelConfig(name="r", vocab_size=200, d_model=32, n_layers=2, n_heads=2, ffn_dim=64, max_seq_len=32,
                      attn=AttentionConfig(kind="gqa", n_kv_heads=1), moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=32))
    tc = TrainConfig(lr=3e-3, warmup_steps=0, max_steps=6)
    batch = lambda step: synthetic_batch(2, 16, 200, seed=1, step=step)

    ref = Trainer(build_model(cfg, device="cpu", seed=0), tc)
    for s in range(6):
        ref.step(*batch(s))

    d = str(tmp_path / "ck")
    t1 = Trainer(build_model(cfg, device="cpu", seed=0), tc)
    with pytest.raises(InjectedFault):
        train_with_recovery(t1, batch, 6, CheckpointManager(d, keep=2), save_every=2,
                            injector=FaultInjector([FaultSpec(0, 5, "raise")]))
    mgr = CheckpointManager(d, keep=2)
    assert mgr.steps() == [2, 4]
    newest = os.path.join(d, "step_000000004.rank0.pt")
    with open(newest, "r+b") as f:
        f.truncate(os.path.getsize(newest) // 3)
    t2 = Trainer(build_model(cfg, device="cpu", seed=123), tc)
    res = train_with_recovery(t2, batch, 6, mgr, save_every=2)
    assert res["resumed_from"] == 2 and len(res["losses"]) == 4
    for (n, a), b in zip(ref.model.state_dict().items(), t2.model.state_dict().values()):
        torch.testing.assert_close(a, b, atol=1e-6, rtol=1e-6, msg=n)
    assert mgr.steps() == [4, 6]


def test_async_checkpoint_is_a_consistent_snapshot(tmp_path):
    from omnicoder.training.resilience import CheckpointManager
    t = _DPTrainer.__new__(_DPTrainer)
    torch.manual_seed(0)
    t.model, t.step_idx = nn.Linear(8, 4), 3
    want = {k: v.clone() for k, v in t.model.state_dict().items()}
    mgr = CheckpointManager(str(tmp_path), keep=2)
    mgr.save_async(3, t.model, t)
    with torch.no_grad():
        t.model.weight.add_(1.0)                 # training goes on while the file is written
    mgr.wait()
    fresh = _DPTrainer.__new__(_DPTrainer)
    fresh.model, fresh.step_idx = nn.Linear(8, 4), 0
    assert mgr.load_latest(fresh.model, fresh) == 3 and fresh.step_idx == 3
    for k, v in fresh.model.state_dict().items():
        assert torch.equal(v, want[k]), k
    for s in (4, 5):
        mgr.save_async(s, t.model, t)
    mgr.wait()
    assert mgr.steps() == [4, 5]


def test_leave_survives_a_dead_store():
    """A rank unwinding from a RankFailure after the store host is gone keeps its own exception:
    leave() reports False instead of raising the store's network error."""
    from omnicoder.parallel.health import Heartbeat

    class DeadStore:
        def set(self, key, value):
            raise dist.DistNetworkError("Broken pipe")

    hb = Heartbeat(store=DeadStore(), rank=1, world=3, interval=0.1, timeout=1.0)
    assert hb.leave("RankFailure: rank 2") is False
