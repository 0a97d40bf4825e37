"""Memory-bound / routing / loss / optimiser kernels against their PyTorch oracles."""
import pytest
import torch
import torch.nn.functional as F

from omnicoder import ops
from omnicoder.ops.gemm import interleave_gate_up

pytestmark = pytest.mark.gpu


def _rel(a, b):
    b = b.to(a.device)
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


@pytest.mark.parametrize("rows,dim", [(300, 512), (1000, 2048), (77, 1024), (64, 384)])
def test_rmsnorm_residual_fwd_bwd(cuda_ext, rows, dim):
    torch.manual_seed(0)
    x = torch.randn(rows, dim, device="cuda").to(torch.bfloat16).requires_grad_()
    r = torch.randn(rows, dim, device="cuda").to(torch.bfloat16).requires_grad_()
    w = (1 + 0.1 * torch.randn(dim, device="cuda")).to(torch.bfloat16).requires_grad_()
    y, h = ops.rms_norm(x, w, 1e-6, residual=r)
    xf, rf, wf = (t.detach().float().requires_grad_() for t in (x, r, w))
    hf = xf + rf
    yf = hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-6) * wf
    assert _rel(y, yf) < 1e-2 and _rel(h, hf) < 1e-2
    dy, dh = torch.randn_like(y), torch.randn_like(h)
    torch.autograd.backward([y, h], [dy, dh])
    torch.autograd.backward([yf, hf], [dy.float(), dh.float()])
    assert _rel(x.grad, xf.grad) < 2e-2 and _rel(w.grad, wf.grad) < 2e-2 and _rel(r.grad, rf.grad) < 2e-2


def test_layernorm_fwd_bwd(cuda_ext):
    torch.manual_seed(1)
    x = torch.randn(130, 256, device="cuda").to(torch.bfloat16).requires_grad_()
    w = torch.randn(256, device="cuda").to(torch.bfloat16).requires_grad_()
    b = torch.randn(256, device="cuda").to(torch.bfloat16).requires_grad_()
    y = ops.layer_norm(x, w, b, 1e-5)
    xf, wf, bf = (t.detach().float().requires_grad_() for t in (x, w, b))
    yf = F.layer_norm(xf, (256,), wf, bf, 1e-5)
    assert _rel(y, yf) < 1e-2
    dy = torch.randn_like(y)
    y.backward(dy)
    yf.backward(dy.float())
    assert _rel(x.grad, xf.grad) < 2e-2 and _rel(w.grad, wf.grad) < 2e-2 and _rel(b.grad, bf.grad) < 2e-2


@pytest.mark.parametrize("interleaved", [False, True])
def test_rope_matches_oracle(cuda_ext, interleaved):
    torch.manual_seed(2)
    tab = ops.RopeTable(64, 512, 10000.0, 1.0)
    x = torch.randn(256, 4, 192, device="cuda").to(torch.bfloat16)
    pos = torch.randint(0, 512, (256,), device="cuda")
    ref = ops.apply_rope(x.cpu().float(), tab, pos.cpu(), off=128, interleaved=interleaved)
    out = ops.apply_rope(x.clone(), tab, pos, off=128, interleaved=interleaved)
    assert _rel(out, ref) < 1e-2


def test_embedding_fwd_bwd(cuda_ext):
    torch.manual_seed(3)
    w = torch.randn(1000, 256, device="cuda").to(torch.bfloat16).requires_grad_()
    ids = torch.randint(0, 1000, (512,), device="cuda")
    y = ops.embedding(ids, w)
    assert torch.equal(y, w.detach()[ids])
    dy = torch.randn_like(y)
    y.backward(dy)
    ref = torch.zeros(1000, 256, device="cuda").index_add_(0, ids, dy.float())
    assert _rel(w.grad, ref) < 1e-2


def test_lm_head_cross_entropy(cuda_ext):
    torch.manual_seed(4)
    h = torch.randn(600, 256, device="cuda").to(torch.bfloat16).requires_grad_()
    w = (0.05 * torch.randn(32000, 256, device="cuda")).to(torch.bfloat16).requires_grad_()
    lab = torch.randint(0, 32000, (600,), device="cuda")
    lab[7] = -100
    loss = ops.lm_head_cross_entropy(h, w, lab, chunk=256)
    hf, wf = h.detach().float().requires_grad_(), w.detach().float().requires_grad_()
    ref = F.cross_entropy(hf @ wf.t(), lab, ignore_index=-100)
    assert abs(loss.item() - ref.item()) < 2e-2
    loss.backward()
    ref.backward()
    assert _rel(h.grad, hf.grad) < 3e-2 and _rel(w.grad, wf.grad) < 3e-2


def test_adamw_matches_torch(cuda_ext):
    torch.manual_seed(5)
    p = torch.nn.Parameter(torch.randn(1003, device="cuda").to(torch.bfloat16))
    ref = torch.nn.Parameter(p.detach().float().clone())
    opt = ops.FusedAdamW([p], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, no_decay_1d=False)
    topt = torch.optim.AdamW([ref], lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1)
    for _ in range(3):
        g = torch.randn(1003, device="cuda").to(torch.bfloat16)
        p.grad = g
        ref.grad = g.float()
        opt.step()
        topt.step()
    assert _rel(opt.state[0]["master"], ref.detach()) < 1e-5
    assert _rel(p, ref.detach()) < 1e-2


@pytest.mark.parametrize("capacity", [0, 40])
def test_moe_matches_oracle(cuda_ext, capacity):
    torch.manual_seed(6)
    T, D, E, Fd, K = 256, 256, 8, 128, 2
    x = torch.randn(T, D, device="cuda").to(torch.bfloat16).requires_grad_()
    rw = (0.1 * torch.randn(E, D, device="cuda")).to(torch.bfloat16).requires_grad_()
    w1 = 0.05 * torch.randn(E, Fd, D, device="cuda")
    w3 = 0.05 * torch.randn(E, Fd, D, device="cuda")
    w13 = interleave_gate_up(w1, w3).to(torch.bfloat16).requires_grad_()
    w2 = (0.05 * torch.randn(E, D, Fd, device="cuda")).to(torch.bfloat16).requires_grad_()
    add = torch.randn(T, D, device="cuda").to(torch.bfloat16).requires_grad_()
    out, aux = ops.moe_ffn(x, rw, w13, w2, K, capacity, True, 0.01, 0.001, add=add)
    xs = [t.detach().float().requires_grad_() for t in (x, rw, w13, w2, add)]
    ref, aux_ref = ops.moe_ffn_torch(xs[0], xs[1], xs[2], xs[3], K, capacity, True, 0.01, 0.001, add=xs[4])
    assert _rel(out, ref) < 2e-2
    assert abs(aux.item() - aux_ref.item()) < 1e-3
    dout = torch.randn_like(out)
    out.backward(dout)
    (ref * dout.float()).sum().add(aux_ref).backward()
    for got, want, name in zip((x, rw, w13, w2, add), xs, ("x", "router", "w13", "w2", "add")):
        assert _rel(got.grad, want.grad) < 5e-2, name


def test_swiglu_mlp_matches_oracle(cuda_ext):
    torch.manual_seed(7)
    x = torch.randn(300, 256, device="cuda").to(torch.bfloat16).requires_grad_()
    w13 = (0.05 * torch.randn(2 * 384, 256, device="cuda")).to(torch.bfloat16).requires_grad_()
    w2 = (0.05 * torch.randn(256, 384, device="cuda")).to(torch.bfloat16).requires_grad_()
    res = torch.randn(300, 256, device="cuda").to(torch.bfloat16).requires_grad_()
    y = ops.swiglu_mlp(x, w13, w2, residual=res)
    xs = [t.detach().float().requires_grad_() for t in (x, w13, w2, res)]
    yr = ops.swiglu_mlp(*[t.cpu() for t in xs[:3]], residual=xs[3].cpu())
    assert _rel(y, yr) < 2e-2


def _plan_reference(idx, E, capacity, align):
    """Token-order ranks inside each expert, kept while rank < capacity, segments padded to align."""
    flat = idx.flatten().tolist()
    seen = [0] * E
    ranks = []
    for e in flat:
        ranks.append(seen[e])
        seen[e] += 1
    kept = [min(c, capacity) if capacity > 0 else c for c in seen]
    offsets = [0]
    for e in range(E):
        offsets.append(offsets[-1] + (kept[e] + align - 1) // align * align)
    pos = [offsets[e] + r if r < kept[e] else -1 for e, r in zip(flat, ranks)]
    src = [-1] * offsets[-1]
    for i, p in enumerate(pos):
        if p >= 0:
            src[p] = i
    return seen, offsets, pos, src


@pytest.mark.parametrize("T,K,E,cap,align", [(64, 4, 32, 0, 1), (200, 4, 32, 20, 1), (100, 6, 64, 0, 128), (5, 2, 8, 1, 128)])
def test_small_permutation_plan_matches_reference(cuda_ext, T, K, E, cap, align):
    """T * K <= 1024 pairs: the one-CTA plan kernel gives the stable token-order permutation."""
    g = torch.Generator().manual_seed(T + E)
    idx = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(T)]).to(torch.int32).cuda()
    counts_r, offsets_r, pos_r, src_r = _plan_reference(idx.cpu(), E, cap, align)
    rows = offsets_r[-1]
    counts, offsets, pos, src = cuda_ext.moe_plan(idx, E, cap, rows, align)
    torch.cuda.synchronize()
    assert counts.tolist() == counts_r and offsets.tolist() == offsets_r
    assert pos.flatten().tolist() == pos_r and src.tolist() == src_r


def test_adamw_multi_tensor_with_clip_matches_torch(cuda_ext):
    """Many small parameters (multi-tensor kernels) and large ones (one launch each), with the
    device-side global-norm clip, against torch.optim.AdamW + clip_grad_norm_."""
    torch.manual_seed(7)
    shapes = [(2048,), (33,), (512, 300), (1 << 20 | 8,), (64, 2048), (7,)] + [(2048,)] * 60
    ps = [torch.nn.Parameter(torch.randn(s, device="cuda").to(torch.bfloat16)) for s in shapes]
    refs = [torch.nn.Parameter(p.detach().float().clone()) for p in ps]
    opt = ops.FusedAdamW(ps, lr=1e-2, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=0.5)
    topt = torch.optim.AdamW([{"params": [r for r in refs if r.dim() > 1], "weight_decay": 0.1},
                              {"params": [r for r in refs if r.dim() <= 1], "weight_decay": 0.0}],
                             lr=1e-2, betas=(0.9, 0.95))
    for _ in range(3):
        for p, r in zip(ps, refs):
            g = torch.randn(p.shape, device="cuda").to(torch.bfloat16)
            p.grad, r.grad = g, g.float()
        opt.step()
        torch.nn.utils.clip_grad_norm_(refs, 0.5)
        topt.step()
    for i, r in enumerate(refs):
        assert _rel(opt.state[i]["master"], r.detach()) < 1e-4, i
        assert _rel(ps[i], r.detach()) < 1e-2, i
