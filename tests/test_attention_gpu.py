"""tcgen05 flash attention (forward + backward) against the fp32 PyTorch oracle."""
import math

import pytest
import torch

from omnicoder.ops.attention import attention, attention_torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


CASES = [
    # name, B, S, H, Hk, Dk, Dr, Dv, window
    ("mha64", 2, 256, 4, 4, 64, 0, 64, 0),
    ("mha128", 1, 384, 2, 2, 128, 0, 128, 0),
    ("gqa128", 1, 256, 8, 2, 128, 0, 128, 0),
    ("mla192", 2, 256, 4, 4, 128, 64, 128, 0),
    ("mla192_window", 1, 512, 2, 2, 128, 64, 128, 200),
    ("gqa_window", 1, 512, 4, 2, 128, 0, 128, 128),
]


@pytest.mark.parametrize("name,B,S,H,Hk,Dk,Dr,Dv,window", CASES)
def test_attention_fwd_bwd(cuda_ext, name, B, S, H, Hk, Dk, Dr, Dv, window):
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
    o = attention(q, k, v, kr, seq=S, causal=True, window=window, scale=scale)
    ref = attention_torch(q.float(), k.float(), v.float(), None if kr is None else kr.float(), seq=S, causal=True,
                          window=window, scale=scale)
    assert _rel(o, ref) < 2e-2, "forward"
    do = torch.randn_like(o)
    o.backward(do)
    qf = q.detach().float().requires_grad_()
    kf = k.detach().float().requires_grad_()
    vf = v.detach().float().requires_grad_()
    krf = kr.detach().float().requires_grad_() if kr is not None else None
    r = attention_torch(qf, kf, vf, krf, seq=S, causal=True, window=window, scale=scale)
    r.backward(do.float())
    assert _rel(q.grad, qf.grad) < 3e-2, "dq"
    assert _rel(k.grad, kf.grad) < 3e-2, "dk"
    assert _rel(v.grad, vf.grad) < 3e-2, "dv"
    if kr is not None:
        assert _rel(kr.grad, krf.grad) < 3e-2, "dk_rope"
