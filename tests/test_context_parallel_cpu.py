"""Context-parallel (all-to-all over heads) attention on gloo ranks: the output and
the q / k / v / rope-key gradients of every rank's sequence chunk must equal one
process attending over the whole sequences."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _data(rope: bool, world: int = 2):
    g = torch.Generator().manual_seed(3)
    B, S, H, Hk, Dk, Dv, Dr = 2, 16, 2 * world, world, 8, 8, 4
    T = B * S
    q = torch.randn(T, H, Dk + (Dr if rope else 0), generator=g)
    k = torch.randn(T, Hk, Dk, generator=g)
    v = torch.randn(T, Hk, Dv, generator=g)
    kr = torch.randn(T, Dr, generator=g) if rope else None
    dout = torch.randn(T, H, Dv, generator=g)
    return B, S, q, k, v, kr, dout


def _chunk(x, B, S, W, r):
    s = S // W
    return x.reshape(B, S, *x.shape[1:])[:, r * s:(r + 1) * s].reshape(B * s, *x.shape[1:])


def _worker(rank, world, port, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from omnicoder.ops.attention import attention_torch
        from omnicoder.parallel.context import context_parallel_attention, gather_sequence, positions, shard_sequence
        worst = 0.0
        for rope in (False, True):
            for window in (0, 5):
                B, S, q, k, v, kr, dout = _data(rope, world)
                full = [t.clone().requires_grad_(True) for t in (q, k, v)] + \
                       ([kr.clone().requires_grad_(True)] if rope else [None])
                ref = attention_torch(*full[:3], full[3], seq=S, causal=True, window=window)
                (ref * dout).sum().backward()
                loc = [_chunk(t, B, S, world, rank).clone().requires_grad_(True) for t in (q, k, v)]
                lkr = _chunk(kr, B, S, world, rank).clone().requires_grad_(True) if rope else None
                out = context_parallel_attention(*loc, lkr, batch=B, causal=True, window=window)
                (out * _chunk(dout, B, S, world, rank)).sum().backward()
                pairs = [(out, _chunk(ref.detach(), B, S, world, rank))]
                pairs += [(a.grad, _chunk(b.grad, B, S, world, rank)) for a, b in zip(loc, full[:3])]
                if rope:
                    pairs.append((lkr.grad, _chunk(full[3].grad, B, S, world, rank)))
                worst = max([worst] + [float((a - b).abs().max()) for a, b in pairs])
        x = torch.arange(2 * 8 * 3, dtype=torch.float32).reshape(2, 8, 3)
        ok = torch.equal(gather_sequence(shard_sequence(x)), x)
        ok &= torch.equal(positions(8), torch.arange(rank * 8 // world, (rank + 1) * 8 // world))
        q_out.put((rank, worst, bool(ok)))
    finally:
        dist.destroy_process_group()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_context_parallel_matches_full_attention(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, worst, ok in res:
        assert worst < 1e-4, (rank, worst)
        assert ok
