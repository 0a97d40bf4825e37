"""Block-scaled fp8 (1 x 128 activations, 128 x 128 weights): the CPU quantisers
round-trip within e4m3 precision; on the GPU the quantisation kernels match the
PyTorch quantisers and the tcgen05 fp8 GEMM (dense and per-expert grouped)
matches an fp32 matmul of the dequantised operands."""
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


@pytest.mark.gpu
def test_fp8_quant_kernels_match_torch():
    from omnicoder.ops import _ext
    C = _ext.load()
    torch.manual_seed(2)
    x = (torch.randn(300, 512, device="cuda") * 2).to(torch.bfloat16)
    xq, sx = C.fp8_quant_act(x)
    rq, rs = fp8.quantize_act_torch(x)
    assert torch.equal(sx, rs)
    assert torch.equal(xq.float(), rq.float())
    w = (torch.randn(2, 260, 384, device="cuda") * 0.02).to(torch.bfloat16)
    wq, sw = C.fp8_quant_weight(w)
    rq, rs = fp8.quantize_weight_torch(w)
    assert torch.equal(sw, rs)
    assert torch.equal(wq.float(), rq.float())


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (256, 384, 512), (300, 520, 1024), (2048, 4096, 4096)])
def test_fp8_gemm_dense(M, N, K):
    torch.manual_seed(3)
    x = torch.randn(M, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(N, K, device="cuda") * 0.02).to(torch.bfloat16)
    wq, sw = fp8.quantize_weight(w)
    y = fp8.fp8_mm(x, wq, sw)
    xq, sx = fp8.quantize_act(x)
    ref = fp8.dequantize_act(xq, sx) @ fp8.dequantize_weight(wq, sw).t()
    assert _rel(y, ref) < 1e-2
    # and against the bf16 product (fp8 quantisation error)
    assert _rel(y, x.float() @ w.float().t()) < 0.08


@pytest.mark.gpu
def test_fp8_gemm_grouped():
    torch.manual_seed(4)
    G, N, K = 4, 256, 384
    counts = [128, 0, 384, 256]
    off = torch.tensor([0, 128, 128, 512, 768], dtype=torch.int32, device="cuda")
    rows = 768
    x = torch.randn(rows, K, device="cuda").to(torch.bfloat16)
    w = (torch.randn(G, N, K, device="cuda") * 0.02).to(torch.bfloat16)
    wq, sw = fp8.quantize_weight(w)
    y = fp8.fp8_grouped_mm(x, wq, sw, off, rows)
    xq, sx = fp8.quantize_act(x)
    xd, wd = fp8.dequantize_act(xq, sx), fp8.dequantize_weight(wq, sw)
    ref = torch.cat([xd[int(off[g]):int(off[g + 1])] @ wd[g].t() for g in range(G)])
    assert _rel(y, ref) < 1e-2
