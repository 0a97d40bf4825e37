"""Tiny MoE LM (4 layers, d 256, 8 heads of 32, RoPE, RMSNorm, 4 SwiGLU experts of ffn 512,
top-2 softmax router, tied 32000 vocab) on CPU in fp32, seed 0: forward, loss, backward,
one AdamW step (lr 1e-3) and a 32-token greedy KV-cache decode from a 16-token prompt,
checked against the independent fp32 oracle (omnicoder.reference_impl) to 1e-4."""
import torch

from omnicoder.config import get_preset
from omnicoder.inference.generate import generate
from omnicoder.models.lm import build_model
from omnicoder.ops import FusedAdamW
from omnicoder.reference_impl import ReferenceLM


def _setup():
    torch.manual_seed(0)
    cfg = get_preset("tiny_moe")
    model = build_model(cfg, device="cpu", seed=0)
    ref = ReferenceLM(cfg, model.state_dict())
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 32000, (2, 128), generator=g)
    labels = torch.randint(0, 32000, (2, 128), generator=g)
    return cfg, model, ref, ids, labels


def test_forward_loss_backward_adamw_match_oracle():
    cfg, model, ref, ids, labels = _setup()
    logits = model(ids, all_logits=True)["logits"]
    assert torch.allclose(logits, ref(ids), atol=1e-4, rtol=0)
    out = model(ids, labels=labels)
    lref = ref.loss(ids, labels)
    assert abs(out["ce"].item() - lref.item()) < 1e-4
    out["loss"].backward()
    lref.backward()
    for name, p in model.named_parameters():
        rp = ref.w(name)
        assert p.grad is not None, name
        assert torch.allclose(p.grad, rp.grad, atol=1e-4, rtol=1e-3), name
    # Adam's first update is ~lr * g / (|g| + eps): on gradients of ~1e-9 the 1e-8-level
    # summation-order noise of two implementations flips signs, so the optimisers are
    # compared on identical gradients (the model's), and the models after the step.
    for name, p in model.named_parameters():
        ref.w(name).grad = p.grad.detach().clone()
    opt = FusedAdamW(model.parameters(), lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01,
                     no_decay_1d=False)
    names = [n for n, _ in model.named_parameters()]
    topt = torch.optim.AdamW([ref.w(n) for n in names], lr=1e-3, betas=(0.9, 0.999), eps=1e-8, weight_decay=0.01)
    opt.step()
    topt.step()
    for name, p in model.named_parameters():
        assert torch.allclose(p.detach(), ref.w(name).detach(), atol=1e-4, rtol=0), name
    # the updated model still agrees with the updated oracle
    assert torch.allclose(model(ids, all_logits=True)["logits"], ref(ids), atol=1e-4, rtol=0)


def test_greedy_kv_cache_decode_matches_oracle():
    cfg, model, ref, _, _ = _setup()
    prompt = torch.randint(0, 32000, (1, 16), generator=torch.Generator().manual_seed(1))
    out = generate(model, prompt, 32, temperature=0.0)
    want = ref.greedy(prompt, 32)
    assert torch.equal(out[:, 16:], want)


def test_batched_decode_equals_full_forward():
    cfg, model, ref, ids, _ = _setup()
    from omnicoder.inference.kv_cache import KVCache

    model.eval()
    cache = KVCache(cfg, 2, 64, "cpu")
    pre = model.forward_cached(ids[:, :20], cache, prefill=True)
    steps = [model.forward_cached(ids[:, i:i + 1], cache) for i in range(20, 40)]
    inc = torch.cat([pre] + steps, dim=1)
    full = model(ids[:, :40], all_logits=True)["logits"]
    assert torch.allclose(inc, full, atol=1e-4, rtol=0)


def test_windowed_decode_and_memory_slots():
    """Sliding-window decode equals the windowed full forward; compressed memory rows
    (segment means of tokens older than the window) are attended after compression."""
    from omnicoder.config import AttentionConfig, ModelConfig
    from omnicoder.inference.kv_cache import KVCache
    from omnicoder.models.lm import build_model

    cfg = ModelConfig(name="win", vocab_size=200, d_model=32, n_layers=2, n_heads=4, ffn_dim=64, max_seq_len=128,
                      attn=AttentionConfig(kind="gqa", n_kv_heads=2, window=8))
    m = build_model(cfg, seed=0).eval()
    ids = torch.randint(0, 200, (2, 40), generator=torch.Generator().manual_seed(3))
    full = m(ids, all_logits=True)["logits"]
    cache = KVCache(cfg, 2, 64, "cpu")
    pre = m.forward_cached(ids[:, :20], cache, prefill=True)
    steps = [m.forward_cached(ids[:, i:i + 1], cache) for i in range(20, 40)]
    assert torch.allclose(torch.cat([pre] + steps, 1), full, atol=1e-4)
    # with 4 memory rows
    cfg.attn.mem_slots = 4
    cache = KVCache(cfg, 2, 64, "cpu")
    m.forward_cached(ids[:, :32], cache, prefill=True)
    assert cache.compress_memory(window=8) == 4
    k_rows = cache.k[0][:, 4:4 + 24].float()
    assert torch.allclose(cache.k[0][:, 0], k_rows[:, :6].mean(1), atol=1e-6)
    with_mem = m.forward_cached(ids[:, 32:33], cache)
    cache.n_mem = 0
    cache.lengths -= 1
    without = m.forward_cached(ids[:, 32:33], cache)
    assert torch.isfinite(with_mem).all() and not torch.allclose(with_mem, without)
