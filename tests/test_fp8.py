"""Block-scaled fp8 (1 x 128 activations, 128 x 128 weights): the CPU quantisers
round-trip within e4m3 precision (power-of-two and exact fp32 scales); on the GPU the
quantisation kernels match the PyTorch quantisers and both GEMM variants (block-scaled
MMA with power-of-two scales, epilogue promotion with fp32 scales; dense and per-expert
grouped) match an fp32 matmul of the dequantised operands, row by row, also when the
scales differ by orders of magnitude between rows, weight blocks and K blocks."""
import pytest
import torch

from omnicoder.ops import fp8


def test_quantisers_round_trip_cpu():
    torch.manual_seed(0)
    x = torch.randn(200, 384) * 3
    xq, sx = fp8.quantize_act_torch(x)
    assert xq.dtype == torch.float8_e4m3fn and sx.shape == (3, 256)
    err = (fp8.dequantize_act(xq, sx) - x).abs() / x.abs().clamp_min(1e-3)
    assert (err < 0.07).float().mean() > 0.99
    w = torch.randn(3, 300, 256) * 0.02
    wq, sw = fp8.quantize_weight_torch(w)
    assert sw.shape == (3, 3, 2)
    assert ((fp8.dequantize_weight(wq, sw) - w).abs().max() / w.abs().max()) < 0.07


@pytest.mark.parametrize("pow2", [True, False])
def test_scales_power_of_two_and_bounded(pow2):
    torch.manual_seed(5)
    x = torch.randn(64, 256) * torch.logspace(-6, 6, 64, base=2.0)[:, None]
    x[3, :128] = 0
    xq, sx = fp8.quantize_act_torch(x, pow2=pow2)
    s = sx[:, :64]
    assert float(s[0, 3]) == 1.0                              # all-zero block
    amax = x.view(64, 2, 128).abs().amax(-1).t()
    assert bool((amax <= s * 448 * (1 + 1e-6)).all())         # no saturation
    m, _ = torch.frexp(s)
    assert bool((m == 0.5).all()) == pow2
    if pow2:
        nz = amax > 0
        assert bool((s[nz] < amax[nz] / 448 * 2).all())          # the smallest power of two that fits


def test_fp8_mm_cpu_matches_dequantised_matmul():
    torch.manual_seed(1)
    x = torch.randn(64, 256)
    w = torch.randn(96, 256) * 0.05
    wq, sw = fp8.quantize_weight(w)
    y = fp8.fp8_mm(x, wq, sw)
    ref = x @ w.t()
    assert ((y - ref).abs().max() / ref.abs().max()) < 0.08


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def _rowrel(a, b):
    """max over rows of (row max-abs error / row max-abs reference)"""
    a, b = a.float(), b.float()
    return ((a - b).abs().amax(-1) / (b.abs().amax(-1) + 1e-30)).max().item()


@pytest.mark.gpu
@pytest.mark.parametrize("pow2", [True, False])
def test_fp8_quant_kernels_match_torch(pow2):
    from omnicoder.ops import _ext
    C = _ext.load()
    torch.manual_seed(2)
    x = (torch.randn(300, 512, device="cuda") * 2).to(torch.bfloat16)
    xq, sx = C.fp8_quant_act(x, pow2)
    rq, rs = fp8.quantize_act_torch(x, pow2)
    assert torch.equal(sx, rs)
    assert torch.equal(xq.float(), rq.float())
    w = (torch.randn(2, 260, 384, device="cuda") * 0.02).to(torch.bfloat16)
    wq, sw = C.fp8_quant_weight(w, pow2)
    rq, rs = fp8.quantize_weight_torch(w, pow2)
    assert torch.equal(sw, rs)
    assert torch.equal(wq.float(), rq.float())


def _spread_operands(M, N, K, spread, dev="cuda"):
    """x rows, weight 128-row blocks and K blocks scaled over 2^-spread .. 2^spread so a scale
    applied to the wrong row / block shows as a large per-row error."""
    g = torch.Generator(device="cpu").manual_seed(M * 7 + N)
    x = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g) * 0.02
    if spread:
        x *= torch.pow(2.0, torch.randint(-spread, spread + 1, (M, 1), generator=g).float())
        x *= torch.pow(2.0, torch.randint(-spread, spread + 1, (1, K // 128), generator=g).float()).repeat_interleave(128, 1)
        nb = (N + 127) // 128
        w *= torch.pow(2.0, torch.randint(-spread, spread + 1, (nb, 1), generator=g).float()).repeat_interleave(128, 0)[:N]
    return x.to(dev, torch.bfloat16), w.to(dev, torch.bfloat16)


@pytest.mark.gpu
@pytest.mark.parametrize("scaled_mma", [True, False])
@pytest.mark.parametrize("M,N,K,spread", [(128, 128, 128, 0), (256, 384, 512, 0), (300, 520, 1024, 0),
                                          (2048, 4096, 4096, 0), (384, 640, 768, 6), (256, 1408, 512, 4)])
def test_fp8_gemm_dense(M, N, K, spread, scaled_mma):
    x, w = _spread_operands(M, N, K, spread)
    wq, sw = fp8.quantize_weight(w, pow2=scaled_mma)
    y = fp8.fp8_mm(x, wq, sw, scaled_mma=scaled_mma)
    xq, sx = fp8.quantize_act(x, pow2=scaled_mma)
    ref = fp8.dequantize_act(xq, sx) @ fp8.dequantize_weight(wq, sw).t()
    assert _rel(y, ref) < 1e-2
    assert _rowrel(y, ref) < 2e-2
    # and against the bf16 product (fp8 quantisation error)
    assert _rel(y, x.float() @ w.float().t()) < 0.08


@pytest.mark.gpu
@pytest.mark.parametrize("scaled_mma", [True, False])
def test_fp8_gemm_grouped(scaled_mma):
    torch.manual_seed(4)
    G, N, K = 4, 384, 384
    off = torch.tensor([0, 128, 128, 512, 768], dtype=torch.int32, device="cuda")
    rows = 768
    x, _ = _spread_operands(rows, N, K, 5)
    w = (torch.randn(G, N, K, device="cuda") * 0.02)
    w *= torch.pow(2.0, torch.arange(G, device="cuda").float() - 2)[:, None, None]
    w = w.to(torch.bfloat16)
    wq, sw = fp8.quantize_weight(w, pow2=scaled_mma)
    y = fp8.fp8_grouped_mm(x, wq, sw, off, rows, scaled_mma=scaled_mma)
    xq, sx = fp8.quantize_act(x, pow2=scaled_mma)
    xd, wd = fp8.dequantize_act(xq, sx), fp8.dequantize_weight(wq, sw)
    ref = torch.cat([xd[int(off[g]):int(off[g + 1])] @ wd[g].t() for g in range(G)])
    assert _rel(y, ref) < 1e-2
    assert _rowrel(y, ref) < 2e-2


def test_fp8_linear_grads_cpu():
    torch.manual_seed(6)
    x = torch.randn(64, 256, requires_grad=True)
    w = (torch.randn(384, 256) * 0.05).requires_grad_()
    y = fp8.fp8_linear(x, w)
    g = torch.randn_like(y)
    y.backward(g)
    xr, wr = x.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    (xr @ wr.t()).backward(g)
    assert _rel(y.detach(), xr.detach() @ wr.detach().t()) < 0.08
    assert _rel(x.grad, xr.grad) < 0.08
    assert _rel(w.grad, wr.grad) < 1e-5            # weight gradient stays high precision
    # the quantised weight is redone after an in-place update (scales double)
    s0 = fp8.WEIGHTS.get(w, False)[1].clone()
    with torch.no_grad():
        w.mul_(2)
    assert torch.equal(fp8.WEIGHTS.get(w, False)[1], 2 * s0)


def test_grouped_swiglu_cpu_fallback():
    torch.manual_seed(7)
    off = torch.tensor([0, 128, 256], dtype=torch.int32)
    x = torch.randn(256, 256)
    w = torch.randn(2, 512, 256) * 0.05
    wq, sw = fp8.quantize_weight(w)
    H, act, aq, sa = fp8.fp8_grouped_swiglu(x, wq, sw, off, 256)
    from omnicoder.ops.gemm import deinterleave_cols
    g, u = deinterleave_cols(H.float())
    a = torch.nn.functional.silu(g) * u
    assert _rel(act, a) < 1e-6
    assert _rel(fp8.dequantize_act(aq, sa), a) < 0.08


@pytest.mark.gpu
def test_fp8_grouped_swiglu_epilogue():
    """The gate|up GEMM's SwiGLU + requantisation epilogue: the pre-activation equals the plain
    epilogue's bit for bit; act and its e4m3 copy match silu(g) * u row by row; scales are powers
    of two that the down GEMM consumes."""
    from omnicoder.ops.gemm import deinterleave_cols
    G, F2, K = 3, 768, 512
    off = torch.tensor([0, 256, 256, 640], dtype=torch.int32, device="cuda")
    rows = 640
    x, _ = _spread_operands(rows, F2, K, 3)
    w = (torch.randn(G, F2, K, device="cuda") * 0.02).to(torch.bfloat16)
    wq, sw = fp8.quantize_weight(w)
    H, act, aq, sa = fp8.fp8_grouped_swiglu(x, wq, sw, off, rows)
    Href = fp8.fp8_grouped_mm(x, wq, sw, off, rows)
    assert torch.equal(H, Href)
    g, u = deinterleave_cols(Href.float())
    a_ref = torch.nn.functional.silu(g) * u
    assert _rowrel(act, a_ref) < 2e-2
    assert _rowrel(fp8.dequantize_act(aq, sa), a_ref) < 0.08
    m, _ = torch.frexp(sa[:, :rows])
    assert bool((m == 0.5).all())
    # the down GEMM on the requantised act equals the one on a fresh quantisation of act
    w2 = (torch.randn(G, 256, F2 // 2, device="cuda") * 0.02).to(torch.bfloat16)
    q2, s2 = fp8.quantize_weight(w2)
    from omnicoder.ops import _ext
    y = torch.empty(rows, 256, device="cuda", dtype=torch.bfloat16)
    _ext.load().fp8_gemm(aq, sa, q2, s2.reshape(-1), y, off, rows)
    # reference: the same quantised operands, dequantised, in fp32
    ad, wd = fp8.dequantize_act(aq, sa), fp8.dequantize_weight(q2, s2)
    y_ref = torch.cat([ad[int(off[g]):int(off[g + 1])] @ wd[g].t() for g in range(G)])
    assert _rowrel(y, y_ref) < 2e-2


def test_weight_cache_redone_after_optimiser_step():
    """FusedAdamW writes parameters without moving their version counters; its step bumps the
    cache generation so the quantised copies are redone."""
    from omnicoder.ops.optim import FusedAdamW
    w = torch.nn.Parameter(torch.randn(128, 128) * 0.05)
    q0 = fp8.WEIGHTS.get(w, False)
    assert fp8.WEIGHTS.get(w, False) is q0
    w.grad = torch.randn_like(w)
    FusedAdamW([w], lr=1e-2).step()
    assert fp8.WEIGHTS.get(w, False) is not q0


@pytest.mark.gpu
def test_fp8_swiglu_mlp_fused_matches_fp32():
    torch.manual_seed(8)
    T, D, F = 512, 256, 384
    x = (torch.randn(T, D, device="cuda")).to(torch.bfloat16).requires_grad_()
    w13 = (torch.randn(2 * F, D, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_()
    w2 = (torch.randn(D, F, device="cuda") * 0.05).to(torch.bfloat16).requires_grad_()
    y = fp8.fp8_swiglu_mlp(x, w13, w2)
    g = torch.randn_like(y)
    y.backward(g)
    from omnicoder.ops.gemm import deinterleave_cols
    # the same chain of quantisations emulated in fp32: tight agreement
    xq, sx = fp8.quantize_act_torch(x.detach())
    q13, s13 = fp8.quantize_weight_torch(w13.detach())
    q2, s2 = fp8.quantize_weight_torch(w2.detach())
    ge, ue = deinterleave_cols(fp8.dequantize_act(xq, sx) @ fp8.dequantize_weight(q13, s13).t())
    aq, sa = fp8.quantize_act_torch(torch.nn.functional.silu(ge) * ue)
    y_emul = fp8.dequantize_act(aq, sa) @ fp8.dequantize_weight(q2, s2).t()
    assert _rowrel(y.detach(), y_emul) < 2e-2
    # and the full-precision MLP within the fp8 quantisation error
    xr, ar, br = (t.detach().float().requires_grad_() for t in (x, w13, w2))
    gg, uu = deinterleave_cols(xr @ ar.t())
    yr = (torch.nn.functional.silu(gg) * uu) @ br.t()
    yr.backward(g.float())
    assert _rel(y.detach(), yr.detach()) < 0.1
    assert ((y.detach().float() - yr).abs().mean() / yr.abs().mean()).item() < 0.1
    assert _rel(x.grad, xr.grad) < 0.1
    assert _rel(w13.grad, ar.grad) < 0.1
    assert _rel(w2.grad, br.grad) < 0.1


def test_transpose_quantiser_cpu():
    torch.manual_seed(9)
    x = torch.randn(256, 200) * torch.logspace(-4, 4, 200, base=2.0)
    xt, st = fp8.quantize_t_torch(x)
    assert xt.shape == (200, 256) and st.shape == (2, 256)
    deq = (xt.float().view(200, 2, 128) * st[:, :200].t()[:, :, None]).view(200, 256).t()
    assert _rowrel(deq.t(), x.t()) < 0.07


@pytest.mark.gpu
def test_fp8_weight_gradient_gemm():
    """Weight gradient dy^T x with both operands quantised per column and 128-token block: the
    transpose quantiser equals the PyTorch one bit for bit and the per-row-scaled GEMM equals an
    fp32 product of the dequantised operands."""
    from omnicoder.ops import _ext
    C = _ext.load()
    T, N, K = 1024, 640, 384
    dy, x = _spread_operands(T, N, N, 0)[0], _spread_operands(T, K, K, 0)[0]
    dy = dy * torch.pow(2.0, torch.randint(-5, 6, (1, N), device="cuda").float()).to(torch.bfloat16)
    x = x * torch.pow(2.0, torch.randint(-5, 6, (T, 1), device="cuda").float()).to(torch.bfloat16)
    for t in (dy, x):
        q, s = C.fp8_quant_t(t)
        rq, rs = fp8.quantize_t_torch(t)
        assert torch.equal(s, rs) and torch.equal(q.float(), rq.float())
    dw = fp8.wgrad_fp8(dy, x)
    dq, ds = fp8.quantize_t_torch(dy)
    xq, xs = fp8.quantize_t_torch(x)
    deq = lambda q, s, n: (q.float().view(n, T // 128, 128) * s[:, :n].t()[:, :, None]).view(n, T)
    ref = deq(dq, ds, N) @ deq(xq, xs, K).t()
    assert _rowrel(dw, ref) < 2e-2
    assert _rel(dw, dy.float().t() @ x.float()) < 0.08


def test_weight_cache_does_not_keep_weights_alive():
    import gc
    import weakref
    w = torch.nn.Parameter(torch.randn(128, 128))
    fp8.WEIGHTS.get(w, False)
    r = weakref.ref(w)
    del w
    gc.collect()
    assert r() is None
    v = torch.nn.Parameter(torch.randn(128, 128))
    fp8.WEIGHTS.get(v, True)                  # drops the dead entry
    assert all(e[1]() is not None for e in fp8.WEIGHTS._d.values())
