"""Compat family against the reference itself.

The unmodified reference (installed under baseline/_ref) builds a tiny
OmniTransformer in a child process (its package is also named `omnicoder`, so it
never shares a process with this one), runs a full-sequence pass and six
cached decode steps, and hands its state_dict and outputs back.  The compat
model loads that state_dict and must reproduce every output to 1e-5.

The reference runs with TorchDynamo disabled: its blocks call torch.compile at
`.to()` time, which fails on this torch version (reference test suite, same
failure), and `.to()` is what rebuilds its expert banks from the loaded
weights."""
import os
import subprocess
import sys
import textwrap

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "baseline", "_ref")

SCRIPT = textwrap.dedent('''
    import sys, torch
    from omnicoder.modeling.transformer_moe import OmniTransformer
    torch.manual_seed(0)
    m = OmniTransformer(vocab_size=1000, n_layers=2, d_model=64, n_heads=4, mlp_dim=128, n_experts=4, top_k=2,
                        max_seq_len=256, kv_latent_dim=32, multi_token=1)
    m = m.to("cpu"); m.eval()
    ids = torch.randint(0, 1000, (2, 20), generator=torch.Generator().manual_seed(1))
    res = {"sd": {k: v.clone() for k, v in m.state_dict().items()}, "ids": ids}
    with torch.no_grad():
        res["full"] = [t if torch.is_tensor(t) else None for t in m(ids)]
        past, cur, steps = None, ids[:1, -1:], []   # the reference decodes one sequence at a time
        for _ in range(6):
            out = m(cur, past_kv=past, use_cache=True)
            steps.append(out[0].clone())
            past = out[1]
            cur = out[0][:, -1].argmax(-1, keepdim=True)
        res["steps"] = steps
    torch.save(res, sys.argv[1])
''')


@pytest.mark.skipif(not os.path.isdir(os.path.join(REF, "omnicoder")), reason="reference not installed")
def test_compat_matches_reference(tmp_path):
    from omnicoder.models.compat import OmniTransformer, load_reference_state_dict

    script = tmp_path / "run_ref.py"
    script.write_text(SCRIPT)
    out = tmp_path / "ref.pt"
    env = {"PATH": os.environ.get("PATH", ""), "HOME": str(tmp_path), "PYTHONPATH": REF, "TORCHDYNAMO_DISABLE": "1",
           "CUDA_VISIBLE_DEVICES": ""}
    r = subprocess.run([sys.executable, str(script), str(out)], cwd=tmp_path, env=env, capture_output=True, text=True,
                       timeout=900)
    assert r.returncode == 0, r.stderr[-3000:]
    ref = torch.load(out)
    m = OmniTransformer(vocab_size=1000, n_layers=2, d_model=64, n_heads=4, mlp_dim=128, n_experts=4, top_k=2,
                        max_seq_len=256, kv_latent_dim=32, multi_token=1)
    rep = load_reference_state_dict(m, ref["sd"])
    assert not rep["unexpected"] and not rep["shape_mismatch"], rep
    m.eval()
    with torch.no_grad():
        full = m(ref["ids"])
        assert len(full) == len(ref["full"])
        for a, b in zip(full, ref["full"]):
            if b is None:
                assert a is None
            else:
                assert torch.allclose(a, b, atol=1e-5, rtol=0), (a - b).abs().max()
        past, cur = None, ref["ids"][:1, -1:]
        for want in ref["steps"]:
            out = m(cur, past_kv=past, use_cache=True)
            assert torch.allclose(out[0], want, atol=1e-5, rtol=0), (out[0] - want).abs().max()
            past = out[1]
            cur = out[0][:, -1].argmax(-1, keepdim=True)


def test_reference_key_normalisation():
    from omnicoder.models.compat import OmniTransformer, load_reference_state_dict

    m = OmniTransformer(vocab_size=100, n_layers=1, d_model=32, n_heads=4, mlp_dim=64, n_experts=2, top_k=1,
                        max_seq_len=64, kv_latent_dim=8)
    sd = {}
    for k, v in m.state_dict().items():
        k2 = k.replace("moe.experts.0.", "moe.experts.0._orig_mod.")
        sd["module." + k2] = v.clone() + 1.0
    sd["module.blocks.0._attn_call._inner.qkv_proj.weight"] = torch.zeros(1)
    sd["module.blocks.0.attn._qkv_compiled.weight"] = torch.zeros(1)
    rep = load_reference_state_dict(m, {"state_dict": sd})
    assert rep["missing"] == [] and rep["unexpected"] == [], rep
    assert torch.allclose(m.blocks[0].moe.experts[0].fc1.weight, sd["module.blocks.0.moe.experts.0._orig_mod.fc1.weight"])


def test_capacity_moe_layer_keeps_ceil_capacity_pairs():
    """transformer_moe.MoELayer's capacity: ceil(T * k / E * cf) pairs per expert (or a static
    capacity); with a capacity at least T the layer equals the dropless computation, and a small
    static capacity drops pairs past it."""
    from omnicoder.models.compat import CapacityMoELayer, CompatConfig, MoELayer
    c = CompatConfig(d_model=32, mlp_dim=64, n_experts=4, top_k=2)
    torch.manual_seed(0)
    layer = CapacityMoELayer(c, capacity_factor=1.2).eval()
    assert layer.expert_capacity(10) == 6          # 10 * 2 / 4 * 1.2 = 6.0
    assert layer.expert_capacity(11) == 7          # 6.6 -> 7
    x = torch.randn(1, 16, 32)
    big = CapacityMoELayer(c, static_capacity=10 ** 6).eval()
    big.load_state_dict(layer.state_dict())
    ref = MoELayer(c).eval()
    ref.load_state_dict(layer.state_dict())
    ref.expert_capacity = lambda n: 10 ** 6
    torch.testing.assert_close(big(x), ref(x))
    one = CapacityMoELayer(c, static_capacity=1).eval()
    one.load_state_dict(layer.state_dict())
    y1, yb = one(x), big(x)
    assert not torch.allclose(y1, yb)              # pairs past one per expert are dropped
    zero_rows = (y1.abs().sum(-1) == 0).sum().item()
    assert zero_rows >= 16 - 4                     # at most 4 experts x 1 pair reach the output
