"""tcgen05 flash attention (forward + backward) against the fp32 PyTorch oracle."""
import math

import pytest
import torch

from omnicoder.ops.attention import attention, attention_torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def _rowrel(a, b):
    """Per-row relative error ||a - b|| / ||b|| over the last dim: (mean, 99th percentile).  A wrong
    small-magnitude region, which the max-abs / max-ref ratio can hide, shows up here at ~1."""
    a, b = a.float().reshape(-1, a.shape[-1]), b.float().reshape(-1, b.shape[-1])
    r = (a - b).norm(dim=-1) / (b.norm(dim=-1) + 1e-6)
    return r.mean().item(), torch.quantile(r, 0.99).item()


def _check_rows(a, b, what):
    mean, p99 = _rowrel(a, b)
    assert mean < 3e-2 and p99 < 1e-1, (what, mean, p99)


CASES = [
    # name, B, S, H, Hk, Dk, Dr, Dv, window
    ("mha64", 2, 256, 4, 4, 64, 0, 64, 0),
    ("mha128", 1, 384, 2, 2, 128, 0, 128, 0),
    ("gqa128", 1, 256, 8, 2, 128, 0, 128, 0),
    ("mla192", 2, 256, 4, 4, 128, 64, 128, 0),
    ("mla192_window", 1, 512, 2, 2, 128, 64, 128, 200),
    ("gqa_window", 1, 512, 4, 2, 128, 0, 128, 128),
]


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("name,B,S,H,Hk,Dk,Dr,Dv,window", CASES)
def test_attention_fwd_bwd(cuda_ext, name, B, S, H, Hk, Dk, Dr, Dv, window, causal):
    torch.manual_seed(0)
    T = B * S
    Dq = Dk + Dr
    dev = "cuda"
    q = torch.randn(T, H, Dq, device=dev).to(torch.bfloat16).requires_grad_()
    # k and v as strided views of one buffer, like the MLA up-projection output
    kv = torch.randn(T, Hk, Dk + Dv, device=dev).to(torch.bfloat16)
    k = kv[:, :, :Dk].detach().requires_grad_()
    v = kv[:, :, Dk:].detach().requires_grad_()
    kr = torch.randn(T, Dr, device=dev).to(torch.bfloat16).requires_grad_() if Dr else None
    scale = 1.0 / math.sqrt(Dq)
    o = attention(q, k, v, kr, seq=S, causal=causal, window=window, scale=scale)
    ref = attention_torch(q.float(), k.float(), v.float(), None if kr is None else kr.float(), seq=S, causal=causal,
                          window=window, scale=scale)
    assert _rel(o, ref) < 2e-2, "forward"
    do = torch.randn_like(o)
    o.backward(do)
    qf = q.detach().float().requires_grad_()
    kf = k.detach().float().requires_grad_()
    vf = v.detach().float().requires_grad_()
    krf = kr.detach().float().requires_grad_() if kr is not None else None
    r = attention_torch(qf, kf, vf, krf, seq=S, causal=causal, window=window, scale=scale)
    r.backward(do.float())
    assert _rel(q.grad, qf.grad) < 3e-2, "dq"
    assert _rel(k.grad, kf.grad) < 3e-2, "dk"
    assert _rel(v.grad, vf.grad) < 3e-2, "dv"
    _check_rows(o, ref, "o")
    _check_rows(q.grad, qf.grad, "dq")
    _check_rows(v.grad, vf.grad, "dv")
    if not (window and causal):
        # with a causal window the last keys of a sequence see few queries; their dk rows are tiny
        _check_rows(k.grad, kf.grad, "dk")
    if kr is not None:
        assert _rel(kr.grad, krf.grad) < 3e-2, "dk_rope"


def test_attention_kv_single_gradient_matches_views():
    """attention_kv (keys/values as column blocks of one tensor, one gradient buffer) gives
    the gradients of attention() on the two views."""
    from omnicoder.ops import attention, attention_kv
    torch.manual_seed(3)
    T, H, dn, dr, dv, seq = 512, 4, 128, 64, 128, 256
    q = (torch.randn(T, H, dn + dr, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_()
    kv = (torch.randn(T, H, dn + dv, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_()
    kr = (torch.randn(T, dr, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_()
    g = torch.randn(T, H, dv, device="cuda").to(torch.bfloat16)
    o1 = attention_kv(q, kv, dn, kr, seq=seq, causal=True)
    o1.backward(g)
    grads1 = [t.grad.clone() for t in (q, kv, kr)]
    for t in (q, kv, kr):
        t.grad = None
    o2 = attention(q, kv[:, :, :dn], kv[:, :, dn:], kr, seq=seq, causal=True)
    o2.backward(g)
    assert torch.equal(o1, o2)
    for a, t in zip(grads1, (q, kv, kr)):
        assert torch.equal(a, t.grad)
