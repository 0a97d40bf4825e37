"""torch.ops.omnicoder dispatcher operators, the MLA provider registry and the
4-bit linear swap.  Oracles: fp32 PyTorch attention and unpack-dequantise-matmul."""
import math

import pytest
import torch
import torch.nn as nn

from omnicoder.ops import _ext
from omnicoder.quant.int4 import dequant_int4, pack_int4

needs_ext = pytest.mark.skipif(not _ext.available(), reason="extension not built")


def _attn_ref(q, k, v, mask=None, causal=False):
    s = q.float() @ k.float().transpose(-1, -2) / math.sqrt(q.shape[-1])
    if causal:
        T = q.shape[1]
        s = s.masked_fill(torch.ones(T, T, dtype=torch.bool, device=q.device).triu(1), float("-inf"))
    if mask is not None:
        s = s.masked_fill(~mask, float("-inf")) if mask.dtype == torch.bool else s + mask.float()
    return torch.softmax(s, -1) @ v.float()


def _int4_ref(x, packed, scale, K, zero):
    nib = dequant_int4(packed, torch.ones_like(scale), K, offset=0.0)            # raw nibbles
    w = (nib - zero.float().reshape(-1, 1)) * scale.float()[:, None]
    return x.float() @ w.t()


@needs_ext
@pytest.mark.parametrize("causal", [False, True])
def test_mla_cpu(causal):
    from omnicoder.ops.library import mla
    torch.manual_seed(0)
    q, k, v = torch.randn(4, 12, 16), torch.randn(4, 12, 16), torch.randn(4, 12, 8)
    torch.testing.assert_close(mla(q, k, v, None, causal), _attn_ref(q, k, v, causal=causal), atol=1e-5, rtol=1e-5)
    mask = torch.rand(12, 12) > 0.3
    mask[:, 0] = True
    torch.testing.assert_close(mla(q, k, v, mask), _attn_ref(q, k, v, mask=mask), atol=1e-5, rtol=1e-5)


@needs_ext
def test_matmul_int4_cpu_offset_and_zero():
    from omnicoder.ops.library import matmul_int4
    torch.manual_seed(0)
    w = torch.randn(24, 70)
    packed, scale, _ = pack_int4(w)
    x = torch.randn(3, 70)
    torch.testing.assert_close(matmul_int4(x, packed, scale, None, 7.0), x @ dequant_int4(packed, scale, 70, 7.0).t(),
                               atol=1e-4, rtol=1e-4)
    zero = torch.randint(6, 10, (24,)).float()
    torch.testing.assert_close(matmul_int4(x, packed, scale, zero), _int4_ref(x, packed, scale, 70, zero), atol=1e-4,
                               rtol=1e-4)


def test_mla_provider_registry():
    from omnicoder.ops import library
    assert library.resolve_mla_provider("dml") is library.resolve_mla_provider("cpu")
    assert library.resolve_mla_provider(device="cuda") is library.mla
    with pytest.raises(KeyError):
        library.resolve_mla_provider("no-such-backend")
    library.register_mla_provider("double", lambda q, k, v, m, c: 2 * library._cpu_mla(q, k, v, m, c))
    q = torch.randn(2, 5, 8)
    torch.testing.assert_close(library.resolve_mla_provider("double")(q, q, q, None, True),
                               2 * _attn_ref(q, q, q, causal=True))


def test_replace_linears_4bit():
    from omnicoder.ops.library import replace_linears_4bit
    from omnicoder.quant.int4 import Int4Linear
    torch.manual_seed(0)
    net = nn.Sequential(nn.Linear(64, 32), nn.GELU(), nn.Linear(32, 16))
    x = torch.randn(5, 64)
    ref = net(x)
    assert replace_linears_4bit(net) == 2
    assert all(isinstance(net[i], Int4Linear) for i in (0, 2))
    assert (net(x) - ref).norm() < 0.15 * ref.norm()


@pytest.mark.gpu
@pytest.mark.parametrize("D,Dv,causal", [(64, 64, True), (128, 128, False), (128, 128, True)])
def test_mla_cuda_kernel(cuda_ext, D, Dv, causal):
    from omnicoder.ops.library import mla
    torch.manual_seed(0)
    BH, T = 6, 256
    q = torch.randn(BH, T, D, device="cuda", dtype=torch.bfloat16)
    k = torch.randn(BH, T, D, device="cuda", dtype=torch.bfloat16)
    v = torch.randn(BH, T, Dv, device="cuda", dtype=torch.bfloat16)
    out = mla(q, k, v, None, causal)
    assert out.shape == (BH, T, Dv) and out.is_contiguous()
    torch.testing.assert_close(out.float(), _attn_ref(q, k, v, causal=causal), atol=2e-2, rtol=2e-2)
    mask = torch.rand(T, T, device="cuda") > 0.2
    mask[:, 0] = True
    torch.testing.assert_close(mla(q, k, v, mask).float(), _attn_ref(q, k, v, mask=mask), atol=2e-2, rtol=2e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("rows", [4, 40])
@pytest.mark.parametrize("use_zero", [False, True])
def test_matmul_int4_cuda(cuda_ext, rows, use_zero):
    from omnicoder.ops.library import matmul_int4
    torch.manual_seed(0)
    N, K = 384, 512
    packed, scale, _ = pack_int4(torch.randn(N, K))
    x = torch.randn(rows, K)
    zero = torch.randint(6, 10, (N,)).float() if use_zero else torch.full((N,), 8.0)
    ref = _int4_ref(x.bfloat16().float(), packed, scale, K, zero)
    out = matmul_int4(x.cuda().bfloat16(), packed.cuda(), scale.cuda(), zero.cuda() if use_zero else None, 8.0)
    assert out.dtype == torch.bfloat16 and out.shape == (rows, N)
    torch.testing.assert_close(out.float().cpu(), ref, atol=0.05 * ref.abs().max().item(), rtol=2e-2)
