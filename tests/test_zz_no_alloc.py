"""Allocation-free MoE permutation plan, called through its exported C symbol.

Some callers of this library cannot allocate device memory while they run
(for example a plugin inside another runtime that owns all device memory);
`omni_moe_permute_plan_noalloc` serves them with a fixed device scratch array.
This test loads the symbol with ctypes and checks, on two calls in a row with
different routing, that it returns exactly what the regular allocating binding
(`omnicoder._C.moe_plan`) returns, and that oversized problems are refused.
It lives in its own file that pytest collects last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

OK, TOO_LARGE = 0, 1


def _entry():
    import omnicoder._C as C

    lib = ctypes.CDLL(C.__file__)
    f = lib.omni_moe_permute_plan_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p,
                  ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    return f


def _route(T, K, E, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    if T == 0:
        return torch.empty(0, K, dtype=torch.int32, device="cuda")
    # distinct experts per token, like a top-k router
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32)
    return idx.cuda().contiguous()


def test_noalloc_plan_matches_allocating_binding(cuda_ext):
    from omnicoder.ops.moe import cap_rows_for

    f = _entry()
    stream = torch.cuda.current_stream().cuda_stream
    # multi-block problems, then a one-block problem (T*K <= 1024, where the allocating
    # binding switches to its single-CTA kernel) with a capacity, then no tokens at all
    for call, (T, K, E, cap) in enumerate([(3000, 4, 32, 0), (2500, 6, 64, 300), (100, 4, 16, 20), (0, 4, 16, 0)]):
        idx = _route(T, K, E, seed=100 + call)
        rows = cap_rows_for(T, K, E, cap)
        ref_counts, ref_offsets, ref_pos, ref_src = cuda_ext.moe_plan(idx, E, cap, rows)
        counts = torch.full((E,), -7, dtype=torch.int32, device="cuda")
        offsets = torch.full((E + 1,), -7, dtype=torch.int32, device="cuda")
        pos = torch.full((max(T, 1), K), -7, dtype=torch.int32, device="cuda")
        src = torch.full((max(rows, 1),), -7, dtype=torch.int32, device="cuda")
        rc = f(idx.data_ptr() if T else pos.data_ptr(), T, K, E, cap, counts.data_ptr(), offsets.data_ptr(),
               pos.data_ptr(), src.data_ptr(), rows, stream)
        assert rc == OK, f"call {call}: return code {rc}"
        torch.cuda.synchronize()
        assert torch.equal(counts, ref_counts), call
        assert torch.equal(offsets, ref_offsets), call
        assert torch.equal(pos[:T], ref_pos.view(T, K)), call
        used = int(ref_offsets[-1])
        assert torch.equal(src[:used], ref_src[:used]), call


def test_noalloc_plan_rejects_oversized_problem(cuda_ext):
    f = _entry()
    T, K, E = 200_000, 8, 256  # needs 2 * 1563 * 256 scratch integers > 65536
    idx = torch.zeros(1, dtype=torch.int32, device="cuda")
    buf = torch.zeros(16, dtype=torch.int32, device="cuda")
    rc = f(idx.data_ptr(), T, K, E, 0, buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), buf.data_ptr(), 16,
           torch.cuda.current_stream().cuda_stream)
    assert rc == TOO_LARGE
