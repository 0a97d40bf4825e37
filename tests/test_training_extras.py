"""LoRA adapters, distillation, MTP-head training, GRPO / PPO steps and the
programmatic rewards (code runs in a sandboxed child process)."""
import torch

from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig
from omnicoder.models.lm import build_model


def _cfg(**kw):
    c = ModelConfig(name="x", vocab_size=64, d_model=32, n_layers=2, n_heads=4, ffn_dim=64, max_seq_len=64,
                    attn=AttentionConfig(kind="mha"), moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=32))
    for k, v in kw.items():
        setattr(c, k, v)
    return c


def test_lora_trains_only_adapters_and_merges():
    from omnicoder.training.lora import inject_lora, lora_state_dict, merge_lora
    m = build_model(_cfg(), seed=0)
    base = {k: v.clone() for k, v in m.state_dict().items()}
    n = inject_lora(m, r=4, alpha=8)
    assert n > 0
    ids = torch.randint(0, 64, (2, 16), generator=torch.Generator().manual_seed(0))
    opt = torch.optim.AdamW([p for p in m.parameters() if p.requires_grad], lr=1e-2)
    losses = []
    for _ in range(15):
        loss = m(ids, labels=ids)["loss"]
        loss.backward()
        opt.step()
        opt.zero_grad()
        losses.append(float(loss))
    assert losses[-1] < losses[0]
    assert len(lora_state_dict(m)) == 2 * n
    out = m(ids, all_logits=True)["logits"]
    merge_lora(m)
    assert torch.allclose(m(ids, all_logits=True)["logits"], out, atol=1e-4)
    sd = m.state_dict()
    assert any(not torch.equal(sd[k], base[k]) for k in base if k in sd)


def test_distill_and_mtp_heads():
    from omnicoder.training.data import SyntheticTokens, batches
    from omnicoder.training.distill import distill_step, kd_loss, train_mtp_heads
    t = build_model(_cfg(), seed=0).eval()
    s = build_model(_cfg(n_layers=1), seed=1)
    ids = torch.randint(0, 64, (2, 16))
    lt = t(ids, all_logits=True)["logits"]
    assert float(kd_loss(lt, lt, None)) < 1e-5
    opt = torch.optim.AdamW(s.parameters(), lr=1e-2)
    l0 = distill_step(s, t, opt, ids, ids)
    for _ in range(10):
        l1 = distill_step(s, t, opt, ids, ids)
    assert l1 < l0
    m = build_model(_cfg(mtp_heads=2), seed=0)
    fixed = next(batches(SyntheticTokens(64, 16), 2, pin=False))

    def repeat():
        while True:
            yield fixed
    losses = train_mtp_heads(m, repeat(), steps=8, lr=1e-2)
    assert len(losses) == 8 and losses[-1] < losses[0]


def test_rewards_and_sandbox():
    from omnicoder.training.rl import reward_code, reward_exact, reward_numeric
    assert reward_exact(" Paris ", "paris") == 1.0
    assert reward_numeric("so the answer is 42.0", "42") == 1.0 and reward_numeric("41", 42) == 0.0
    good = "def add(a, b):\n    return a + b\n"
    assert reward_code(good, ["assert add(1, 2) == 3", "assert add(-1, 1) == 0"]) == 1.0
    assert reward_code("def add(a, b):\n    return a - b\n", ["assert add(1, 2) == 3", "assert add(1, 0) == 1"]) == 0.5
    assert reward_code("while True:\n    pass\n", ["pass"], timeout_s=1.0) == 0.0


def test_grpo_and_ppo_steps():
    from omnicoder.training.rl import GRPOTrainer, PPOTrainer
    torch.manual_seed(0)
    m = build_model(_cfg(), seed=0)
    ref = build_model(_cfg(), seed=0)
    prompts = torch.randint(0, 64, (2, 4))
    target = 7

    def reward(i, comp):
        return float((comp == target).float().mean())

    g = GRPOTrainer(m, ref, lr=5e-3, group=4, max_new_tokens=6)
    stats = [g.step(prompts, reward) for _ in range(3)]
    assert all(torch.isfinite(torch.tensor(s["loss"])) for s in stats)
    p = PPOTrainer(build_model(_cfg(), seed=2), lr=1e-3, max_new_tokens=6)
    st = p.step(prompts, reward)
    assert torch.isfinite(torch.tensor(st["loss"]))
