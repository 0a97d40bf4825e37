"""Reference-architecture building blocks: router contracts, HRM, memory,
compressive KV, sequence mixers, fast head shortlist (exactness), expert
utilities."""
import torch
import torch.nn as nn

from omnicoder.models.expert_utils import (DiffusionTextGenerator, ExpertPager, HyperExpertSpec,
                                           HyperExpertSynthesizer, PerceiverIOTower, upcycle_ffn_to_experts)
from omnicoder.models.heads import FastHeadShortlist
from omnicoder.models.modules import (HRM, CompressiveKV, ExpertFFN, GatedConvSSM, GatedMambaSSM, GRINGate,
                                      HierarchicalRouter, HyenaMixer1D, InteractionRouter, LandmarkIndexer, LLMRouter,
                                      MultiHeadRouter, RecurrentMemory, TopKRouter, compressive_aux_loss,
                                      load_balance_loss)


def test_router_contracts():
    torch.manual_seed(0)
    x = torch.randn(2, 16, 32)
    for r in (TopKRouter(32, 8, 2), HierarchicalRouter(32, 8, [4, 4], 2), MultiHeadRouter(32, 8, 2), GRINGate(32, 8, 2),
              LLMRouter(32, 8, 2), InteractionRouter(32, 8, 2)):
        idx, scores, probs, aux = r(x)
        assert idx.shape == (2, 16, 2) and scores.shape == (2, 16, 2) and probs.shape == (2, 16, 8)
        assert torch.allclose(scores.sum(-1), torch.ones(2, 16), atol=1e-5)
        assert torch.allclose(probs.sum(-1), torch.ones(2, 16), atol=1e-5)
        assert aux["importance"].shape == (8,)
        assert float(load_balance_loss(aux, 8)) > 0


def test_hierarchical_router_stays_in_group():
    r = HierarchicalRouter(32, 8, [4, 4], 2)
    idx, _, _, _ = r(torch.randn(3, 10, 32))
    g = idx // 4
    assert torch.equal(g[..., 0], g[..., 1])


def test_grin_gate_gradient_flows():
    g = GRINGate(16, 4, 2)
    idx, scores, probs, _ = g(torch.randn(1, 5, 16))
    scores.sum().backward()
    assert g.base_gate.weight.grad is not None


def test_blocks_shapes_and_causality():
    x = torch.randn(2, 24, 32)
    assert HRM(32)(x).shape == x.shape
    assert HRM(32, adaptive_halting=True)(x).shape == x.shape
    mem = RecurrentMemory(32, 4)(x)
    assert mem.shape == (2, 4, 32) and float(compressive_aux_loss(mem, x)) >= 0
    assert LandmarkIndexer(32, 8)(x).shape == (2, 8, 32)
    assert GatedMambaSSM(32)(x).shape == x.shape and GatedConvSSM(32)(x).shape == x.shape
    hy = HyenaMixer1D(32, kernel_size=8)
    y1 = hy(x)
    x2 = x.clone()
    x2[:, 10:] += 1.0
    assert torch.allclose(hy(x2)[:, :10], y1[:, :10], atol=1e-6)       # causal
    km, vm = CompressiveKV(16, 4)(torch.randn(2, 3, 10, 16), torch.randn(2, 3, 10, 16))
    assert km.shape == (2, 3, 4, 16)
    assert ExpertFFN(32, 64)(x).shape == x.shape


def test_fast_head_shortlist_exact():
    torch.manual_seed(0)
    head = nn.Linear(256, 5000)
    fh = FastHeadShortlist.from_linear(head, sub_dims=32)
    h = torch.randn(4, 256)
    assert torch.equal(fh.argmax(h, initial_k=64).squeeze(1), head(h).argmax(-1))


def test_expert_utils():
    class Layer(nn.Module):
        def __init__(self):
            super().__init__()
            self.experts = nn.ModuleList([ExpertFFN(8, 16)])
            self.n_experts = 1
    m = nn.Sequential(Layer())
    assert upcycle_ffn_to_experts(m, 4) == 1 and len(m[0].experts) == 4 and m[0].n_experts == 4
    pager = ExpertPager(capacity=2)
    for i in range(3):
        pager.register(i, lambda: ExpertFFN(8, 16))
    pager.get(0), pager.get(1), pager.get(2), pager.get(2)
    st = pager.stats()
    assert st["evictions"] == 1 and st["hits"] == 1 and len(st["resident"]) == 2
    hx = HyperExpertSynthesizer(HyperExpertSpec(8, 16), cond_dim=4, hidden=32)
    w = hx(torch.randn(2, 4))
    assert w["w1"].shape == (2, 16, 8) and HyperExpertSynthesizer.apply(w, torch.randn(3, 8)).shape == (3, 8)
    assert PerceiverIOTower(d_io=16, d_latent=32, n_latents=4, n_layers=1)(torch.randn(2, 7, 16)).shape == (2, 7, 16)
    emb = torch.randn(50, 16)
    gen = DiffusionTextGenerator(lambda e: e, emb, num_steps=3)
    out = gen.generate(torch.tensor([[1, 2]]), 5, generator=torch.Generator().manual_seed(0))
    assert out.shape == (1, 5) and int(out.max()) < 50
