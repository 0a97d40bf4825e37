"""Split-KV decode attention kernel against the fp32 PyTorch oracle
(omnicoder.ops.decode.decode_attention_torch): MHA, GQA and MLA latent caches,
bf16 and int8 (per-token / per-head scales), single-token and multi-token
(speculative verify) queries, sliding window, ragged cache lengths."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _case(B, Tn, H, Hk, DQ, DV, L, latent, int8, window, seed=0):
    from omnicoder.inference.kv_cache import quantize_int8
    from omnicoder.ops.decode import decode_attention, decode_attention_torch

    dev = torch.device("cuda")
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, Tn, H, DQ, generator=g).to(dev, torch.bfloat16)
    if latent:
        k = torch.randn(B, L, DQ, generator=g).to(dev, torch.bfloat16)
        v = None
    else:
        k = torch.randn(B, L, Hk, DQ, generator=g).to(dev, torch.bfloat16)
        v = torch.randn(B, L, Hk, DV, generator=g).to(dev, torch.bfloat16)
    kv_len = torch.randint(Tn, L + 1, (B,), generator=g).to(dev, torch.int32)
    q_pos = (kv_len[:, None] - Tn + torch.arange(Tn, device=dev)[None, :]).to(torch.int32)
    ks = vs = None
    if int8:
        k, ks = quantize_int8(k, -1)
        if v is not None:
            v, vs = quantize_int8(v, -1)
    scale = 1.0 / math.sqrt(DQ)
    out = decode_attention(q, k, v, q_pos, kv_len, window=window, scale=scale, k_scale=ks, v_scale=vs,
                           latent_v_dim=DV if latent else 0)
    ref = decode_attention_torch(q.float(), k, v, q_pos.long(), kv_len.long(), window=window, scale=scale,
                                 k_scale=ks, v_scale=vs, latent_v_dim=DV if latent else 0)
    torch.cuda.synchronize()
    err = (out.float() - ref.float()).abs().max().item()
    return err, ref.float().abs().max().item()


@pytest.mark.parametrize("int8", [False, True])
@pytest.mark.parametrize("Tn", [1, 5])
@pytest.mark.parametrize("window", [0, 100])
def test_decode_mla_latent(int8, Tn, window):
    err, mag = _case(B=6, Tn=Tn, H=16, Hk=1, DQ=576, DV=512, L=700, latent=True, int8=int8, window=window)
    assert err < 2e-2 * max(1.0, mag), err


@pytest.mark.parametrize("int8", [False, True])
@pytest.mark.parametrize("Tn,H,Hk,D", [(1, 8, 8, 64), (3, 48, 8, 128), (1, 16, 2, 128)])
def test_decode_mha_gqa(int8, Tn, H, Hk, D):
    err, mag = _case(B=5, Tn=Tn, H=H, Hk=Hk, DQ=D, DV=D, L=333, latent=False, int8=int8, window=0)
    assert err < 2e-2 * max(1.0, mag), err


@pytest.mark.parametrize("kind", ["mha", "mla"])
def test_model_incremental_decode_matches_full_forward(kind):
    from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig
    from omnicoder.inference.kv_cache import KVCache
    from omnicoder.models.lm import build_model

    attn = AttentionConfig(kind="mha") if kind == "mha" else AttentionConfig(
        kind="mla", kv_lora_rank=256, qk_rope_dim=64, qk_nope_dim=64, v_head_dim=128)
    cfg = ModelConfig(name="dec", vocab_size=2048, d_model=256, n_layers=2, n_heads=4, ffn_dim=256,
                      tie_embeddings=True, max_seq_len=512, attn=attn,
                      moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=128))
    dev = torch.device("cuda")
    model = build_model(cfg, device=dev, seed=0).eval()
    ids = torch.randint(0, 2048, (2, 256), device=dev)
    with torch.no_grad():
        full = model(ids, all_logits=True)["logits"].float()
        cache = KVCache(cfg, 2, 320, dev)
        pre = model.forward_cached(ids[:, :128], cache, prefill=True)
        steps = [model.forward_cached(ids[:, i:i + 1], cache) for i in range(128, 140)]
    inc = torch.cat([pre] + steps, dim=1).float()
    ref = full[:, :140]
    err = (inc - ref).abs().max().item()
    assert err < 0.05 * ref.abs().max().item(), err


def test_generate_greedy_cuda_runs():
    from omnicoder.config import get_preset
    from omnicoder.inference.generate import generate
    from omnicoder.models.lm import build_model

    cfg = get_preset("tiny_moe")
    dev = torch.device("cuda")
    model = build_model(cfg, device=dev, seed=0).eval()
    prompt = torch.randint(0, 32000, (4, 16), device=dev)
    out = generate(model, prompt, 8, temperature=0.0)
    assert out.shape == (4, 24)
    assert torch.equal(out[:, :16], prompt)


@pytest.mark.parametrize("int8", [False, True])
def test_decode_with_memory_rows(int8):
    """Cache rows [0, n_sink) are visible to every query; token p lives at row sink_rows + p."""
    from omnicoder.inference.kv_cache import quantize_int8
    from omnicoder.ops.decode import decode_attention, decode_attention_torch

    dev = torch.device("cuda")
    g = torch.Generator(device="cpu").manual_seed(1)
    B, Tn, H, DQ, DV, S, L = 4, 2, 16, 576, 512, 64, 600
    q = torch.randn(B, Tn, H, DQ, generator=g).to(dev, torch.bfloat16)
    k = torch.randn(B, S + L, DQ, generator=g).to(dev, torch.bfloat16)
    kv_len = torch.tensor([300, 599, 450, 120], dtype=torch.int32, device=dev)
    q_pos = (kv_len[:, None] - Tn + torch.arange(Tn, device=dev)[None]).to(torch.int32)
    ks = None
    if int8:
        k, ks = quantize_int8(k, -1)
    kw = dict(window=128, scale=1.0 / math.sqrt(DQ), k_scale=ks, latent_v_dim=DV, sink_rows=S, n_sink=60)
    out = decode_attention(q, k, None, q_pos, kv_len, **kw)
    ref = decode_attention_torch(q.float(), k, None, q_pos.long(), kv_len.long(), **kw)
    torch.cuda.synchronize()
    assert (out.float() - ref.float()).abs().max().item() < 2e-2 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("int8", [False, True])
@pytest.mark.parametrize("Tn,H,Hk,D", [(1, 8, 8, 128), (2, 8, 2, 64), (4, 16, 4, 128)])
def test_decode_mha_memory_rows_and_window(int8, Tn, H, Hk, D):
    """Few-row (GEMV) kernel: MHA / GQA caches with memory rows, a window and ragged lengths."""
    from omnicoder.inference.kv_cache import quantize_int8
    from omnicoder.ops.decode import decode_attention, decode_attention_torch

    dev = torch.device("cuda")
    g = torch.Generator(device="cpu").manual_seed(2)
    B, S, L = 5, 16, 700
    q = torch.randn(B, Tn, H, D, generator=g).to(dev, torch.bfloat16)
    k = torch.randn(B, S + L, Hk, D, generator=g).to(dev, torch.bfloat16)
    v = torch.randn(B, S + L, Hk, D, generator=g).to(dev, torch.bfloat16)
    kv_len = torch.tensor([699, 300, 64, 5 + Tn, 513], dtype=torch.int32, device=dev)
    q_pos = (kv_len[:, None] - Tn + torch.arange(Tn, device=dev)[None]).to(torch.int32)
    ks = vs = None
    if int8:
        k, ks = quantize_int8(k, -1)
        v, vs = quantize_int8(v, -1)
    kw = dict(window=200, scale=1.0 / math.sqrt(D), k_scale=ks, v_scale=vs, sink_rows=S, n_sink=12)
    out = decode_attention(q, k, v, q_pos, kv_len, **kw)
    ref = decode_attention_torch(q.float(), k, v, q_pos.long(), kv_len.long(), **kw)
    torch.cuda.synchronize()
    assert (out.float() - ref.float()).abs().max().item() < 2e-2 * max(1.0, ref.abs().max().item())


@pytest.mark.parametrize("mla", [True, False])
@pytest.mark.parametrize("kv", ["int8", "bf16"])
def test_kv_cache_write_kernel_matches_torch(mla, kv):
    """The fused append kernel writes the rows and scales quantize_int8 + index_put would."""
    from omnicoder.inference.kv_cache import quantize_int8
    from omnicoder.ops import _ext
    C = _ext.load()
    dev = torch.device("cuda")
    torch.manual_seed(0)
    B, T, L, sink = 3, 5, 40, 4
    shape = (B, T, 1, 576) if mla else (B, T, 4, 128)
    src = torch.randn(*shape, device=dev).to(torch.bfloat16)
    pos = torch.tensor([[0, 1, 2, 3, 4], [7, 8, 9, 10, 11], [30, 31, 32, 33, 34]], device=dev)
    G, D = shape[2], shape[3]
    dt = torch.int8 if kv == "int8" else torch.bfloat16
    dst = torch.zeros(B, L, G, D, device=dev, dtype=dt)
    sc = torch.zeros(B, L, G, device=dev) if kv == "int8" else None
    C.kv_cache_write(src, pos, dst, sc, sink)
    rows = pos + sink
    b = torch.arange(B, device=dev)[:, None].expand(B, T)
    if kv == "int8":
        q, s = quantize_int8(src, -1)
        assert torch.equal(dst[b, rows], q)
        assert torch.allclose(sc[b, rows], s, rtol=1e-6, atol=0)
    else:
        assert torch.equal(dst[b, rows], src)
    mask = torch.ones(B, L, dtype=torch.bool, device=dev)
    mask[b, rows] = False
    assert (dst[mask] == 0).all()


def test_graphed_decode_matches_eager():
    """A decode step replayed from a CUDA graph produces the eager step's logits and cache."""
    from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig
    from omnicoder.inference.graphs import GraphedStep
    from omnicoder.inference.kv_cache import KVCache
    from omnicoder.models.lm import build_model
    dev = torch.device("cuda")
    attn = AttentionConfig(kind="mla", kv_lora_rank=512, qk_rope_dim=64, qk_nope_dim=64, v_head_dim=128,
                           window=64, mem_slots=8)
    cfg = ModelConfig(name="g", vocab_size=1000, d_model=512, n_layers=2, n_heads=16, ffn_dim=1024,
                      tie_embeddings=True, max_seq_len=512, attn=attn,
                      moe=MoEConfig(n_experts=8, top_k=2, ffn_dim=256, n_shared_experts=1))
    m = build_model(cfg, device=dev, seed=0).eval().prepare_inference()
    B = 4
    ids = torch.randint(0, 1000, (B, 128), device=dev)
    caches = []
    for _ in range(2):
        c = KVCache(cfg, B, 160, dev, kv_dtype="int8")
        with torch.no_grad():
            m.forward_cached(ids, c, prefill=True, last_only=True)
        c.compress_memory(64)
        caches.append(c)
    step = GraphedStep(m, caches[1])
    tok = ids[:, -1]
    for _ in range(4):
        with torch.no_grad():
            le = m.forward_cached(tok[:, None], caches[0])
        lg = step(tok[:, None])
        torch.cuda.synchronize()
        # split-K partial sums of the few-row GEMM are added with fp32 atomics, so two runs
        # may differ in the last bf16 bit of an activation
        assert (le - lg).abs().max().item() < 2e-2 * max(1.0, le.abs().max().item())
        assert torch.equal(caches[0].lengths, caches[1].lengths)
        tok = le[:, -1].argmax(-1)
    assert (caches[0].k[0].float() - caches[1].k[0].float()).abs().max().item() <= 2
