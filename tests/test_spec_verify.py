"""Speculative-decoding verify step (omnicoder.ops.spec): the torch restatement's acceptance
rule and its output distribution on CPU, and the sm_100a kernel against the restatement on GPU."""
import pytest
import torch

from omnicoder.ops.spec import spec_verify, spec_verify_torch


def test_greedy_acceptance_and_rollback():
    V, K = 50, 4
    logits = torch.randn(2, K + 1, V)
    am = logits.argmax(-1)
    draft = am[:, :K].clone()
    draft[0, 2] = (am[0, 2] + 1) % V                  # sequence 0 rejects at position 2
    base = torch.tensor([10, 20], dtype=torch.int32)
    n_acc, nxt, new_len = spec_verify(logits, None, draft, None, base, 0.0)
    assert n_acc.tolist() == [2, K]
    assert nxt.tolist() == [int(am[0, 2]), int(am[1, K])]
    assert new_len.tolist() == [13, 25] and new_len.dtype == torch.int32


def test_rejection_sampling_keeps_target_distribution():
    """The first emitted token (accepted draft or correction) is distributed as p_target."""
    g = torch.Generator().manual_seed(0)
    V, K, N = 6, 1, 20000
    lt = torch.randn(1, K + 1, V, generator=g)
    pt = torch.softmax(lt[0, 0], -1)
    pd = torch.softmax(torch.randn(V, generator=g) * 2, -1)
    counts = torch.zeros(V)
    draws = torch.multinomial(pd, N, replacement=True, generator=g)
    us = torch.rand(N, K + 1, generator=g)
    for i in range(N):
        n_acc, nxt, _ = spec_verify_torch(lt, pd.view(1, 1, V), draws[i].view(1, 1), us[i:i + 1],
                                          torch.zeros(1, dtype=torch.int32), 1.0)
        tok = int(draws[i]) if int(n_acc) == 1 else int(nxt)
        counts[tok] += 1
    assert (counts / N - pt).abs().max() < 0.015


@pytest.mark.gpu
def test_verify_kernel_matches_restatement(cuda_ext):
    g = torch.Generator().manual_seed(1)
    B, K, V = 64, 4, 32000
    for temp in (0.0, 0.7):
        lt = torch.randn(B, K + 1, V, generator=g) * 3
        pd = torch.softmax(torch.randn(B, K, V, generator=g) * 3, -1)
        if temp > 0:
            draft = torch.stack([torch.multinomial(pd[b], 1, generator=g).squeeze(1) for b in range(B)])
        else:
            draft = lt[:, :K].argmax(-1)
            draft[::3, 1] = (draft[::3, 1] + 7) % V      # some sequences reject early
        u = torch.rand(B, K + 1, generator=g)
        base = torch.randint(100, 200, (B,), generator=g, dtype=torch.int32)
        ref = spec_verify_torch(lt, pd if temp > 0 else None, draft, u if temp > 0 else None, base, temp)
        got = spec_verify(lt.cuda(), pd.cuda() if temp > 0 else None, draft.cuda(), u.cuda() if temp > 0 else None,
                          base.cuda(), temp)
        torch.cuda.synchronize()
        assert torch.equal(got[0].cpu(), ref[0]), temp
        assert torch.equal(got[2].cpu(), ref[2]), temp
        same = (got[1].cpu() == ref[1]).float().mean().item()
        assert same == 1.0 if temp == 0 else same >= 0.98, (temp, same)


@pytest.mark.gpu
def test_mtp_self_speculative_on_gpu(cuda_ext):
    """Self-speculative decoding from the MTP heads on the device (verify kernel, few-row projections):
    greedy output equals plain greedy decoding."""
    from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig
    from omnicoder.inference.generate import generate
    from omnicoder.models.lm import build_model
    cfg = ModelConfig(name="mtp_gpu", vocab_size=4096, d_model=512, n_layers=2, n_heads=4, ffn_dim=512,
                      max_seq_len=512, mtp_heads=3,
                      attn=AttentionConfig(kind="mla", kv_lora_rank=256, qk_rope_dim=64, qk_nope_dim=128,
                                           v_head_dim=128),
                      moe=MoEConfig(n_experts=8, top_k=2, ffn_dim=256, n_shared_experts=1))
    m = build_model(cfg, device="cuda", seed=0).eval()
    prompt = torch.randint(1, 4096, (4, 16), generator=torch.Generator().manual_seed(0)).cuda()
    want = generate(m, prompt, 24, temperature=0.0)
    got, st = generate(m, prompt, 24, temperature=0.0, speculative_draft_len=3, mtp_draft=True, return_stats=True)
    assert torch.equal(got, want) and st.proposed_draft_tokens > 0
