"""Quantisation formats: int4 weight-only linear (CPU oracle and the CUDA
GEMV / dequant kernels), per-group u8 / nf4 KV quantisation, paged latent KV."""
import pytest
import torch

from omnicoder.quant import Int4Linear, PagedKvCache, dequant_int4, dequantize_kv, matmul_int4, pack_int4, quantize_kv
from omnicoder.quant.int4 import unpack_int4


def test_int4_pack_roundtrip_and_layout():
    w = torch.randn(16, 70)
    p, s, z = pack_int4(w)
    assert p.shape == (16, 64) and p.dtype == torch.uint8           # 70 -> padded to 128 elements
    q = unpack_int4(p, 70)
    assert int(q.max()) <= 14 and int(q.min()) >= 0
    # low nibble first: element 0 in bits 0-3
    assert torch.equal(p[:, 0] & 0x0F, q[:, 0]) and torch.equal(p[:, 0] >> 4, q[:, 1])
    wd = dequant_int4(p, s, 70, offset=7.0)
    assert (wd - w).abs().max() <= s.max() * 0.5 + 1e-6


def test_int4_linear_close_to_fp32():
    lin = torch.nn.Linear(256, 64)
    q = Int4Linear(lin)
    x = torch.randn(5, 256)
    y, ref = q(x), lin(x)
    assert (y - ref).abs().mean() < 0.1 * ref.abs().mean()


def test_kv_u8_nf4_roundtrip():
    k = torch.randn(2, 4, 9, 100)
    v = torch.randn(2, 4, 9, 100)
    kq, vq, meta = quantize_kv(k, v, "u8", 64)
    kd, vd = dequantize_kv(kq, vq, meta)
    assert kq.dtype == torch.uint8 and kq.shape == k.shape
    assert (kd - k).abs().max() < 0.03 and (vd - v).abs().max() < 0.03
    kq, vq, meta = quantize_kv(k, v, "nf4", 64)
    kd, vd = dequantize_kv(kq, vq, meta)
    assert int(kq.max()) < 16 and torch.isfinite(kd).all()
    assert (kd - k).abs().mean() < 0.35


def test_paged_kv_tail():
    pc = PagedKvCache(page_len=4, max_pages=2)
    k = torch.arange(10.0).view(1, 1, 10, 1)
    pc.append_tokens(k, -k)
    a, b = pc.materialize_tail(5)
    assert a.flatten().tolist() == [5.0, 6.0, 7.0, 8.0, 9.0] and torch.equal(b, -a)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 3, 8, 40])
def test_int4_cuda_matches_cpu(M):
    torch.manual_seed(0)
    w = torch.randn(1000, 512)
    p, s, _ = pack_int4(w)
    x = torch.randn(M, 512).bfloat16()
    ref = matmul_int4(x.float(), p, s, offset=7.0)
    out = matmul_int4(x.cuda(), p.cuda(), s.cuda(), offset=7.0).float().cpu()
    assert (out - ref).abs().max() < 2e-2 * ref.abs().max()
