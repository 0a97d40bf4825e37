"""Inference-side tools: throughput benchmark, kNN-LM cache, batched HTTP
server, GGUF round trip, ONNX decode-step wrappers (numerics vs the models'
own decode paths), decode-step session runner with KV quantisation and paging."""
import json
import os

import pytest
import torch

from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig, get_preset
from omnicoder.models.lm import build_model


def _tiny():
    cfg = ModelConfig(name="t", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=128,
                      attn=AttentionConfig(kind="gqa", n_kv_heads=2), moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=64))
    return cfg, build_model(cfg, device="cpu", seed=0).eval()


def test_benchmarks_run():
    from omnicoder.inference.benchmark import bench_tokens_per_second, decode_benchmark
    cfg, m = _tiny()
    assert bench_tokens_per_second(m, seq_len=8, gen_tokens=4) > 0
    r = decode_benchmark(m, batch=3, prompt_len=8, gen_tokens=5)
    assert r["decode_tokens_per_s"] > 0 and r["p50_tpot_ms"] > 0


def test_knn_cache_blend():
    from omnicoder.inference.knn_cache import KNNCache
    c = KNNCache(dim=8, k=2, lam=0.5)
    h = torch.randn(10, 8)
    c.add(h, torch.arange(10))
    p = c.query(h[3:4], 20)
    assert int(p.argmax()) == 3 and abs(float(p.sum()) - 1) < 1e-5
    lp = c.blend(torch.zeros(1, 20), h[3:4])
    assert int(lp.argmax()) == 3


def test_http_server_batches_requests():
    from fastapi.testclient import TestClient

    from omnicoder.tools.http_server import create_app
    cfg, m = _tiny()
    with TestClient(create_app(m, max_batch=4, batch_window_s=0.05)) as cli:
        assert cli.get("/health").json()["status"] == "ok"
        import concurrent.futures as cf
        with cf.ThreadPoolExecutor(4) as ex:
            outs = list(ex.map(lambda p: cli.post("/generate/text", json={"prompt": p, "max_new_tokens": 3}).json(),
                               ["abcd", "efgh", "ijkl", "mnop"]))
        assert all("text" in o for o in outs)
        h = cli.get("/health").json()
        assert h["served"] == 4 and h["batches"] < 4                  # at least two requests shared a batch
        assert cli.post("/generate/image", json={"prompt": "x"}).status_code == 501   # no decoder given
        assert "/generate/text" in " ".join(cli.get("/").json()["endpoints"])
        assert "<textarea" in cli.get("/ui").text
        met = cli.get("/metrics").text
        assert "omnicoder_requests_served_total 4" in met and "omnicoder_queue_depth" in met
        assert cli.get("/debug/config").json()["config"]["d_model"] == cfg.d_model


def test_gguf_roundtrip(tmp_path):
    from omnicoder.export.gguf import export_model_gguf, read_gguf
    cfg, m = _tiny()
    p = tmp_path / "m.gguf"
    export_model_gguf(m, str(p), dtype="bf16")
    meta, ts = read_gguf(str(p))
    assert meta["general.architecture"] == "omnicoder" and json.loads(meta["omnicoder.config"])["d_model"] == 64
    sd = m.export_state_dict()
    for k, v in sd.items():
        assert torch.allclose(ts[k].float(), v.float(), atol=1e-2, rtol=1e-2), k


def test_onnx_decode_step_wrappers():
    from omnicoder.export.onnx_export import DecodeStepWrapper, io_names
    from omnicoder.inference.kv_cache import KVCache
    from omnicoder.models.compat import OmniTransformer
    # compat family: same tensors as the model's own decode path
    cm = OmniTransformer(vocab_size=100, n_layers=2, d_model=32, n_heads=4, mlp_dim=64, n_experts=2, top_k=1,
                         max_seq_len=64, kv_latent_dim=8).eval()
    w = DecodeStepWrapper(cm)
    ids = torch.tensor([[5]])
    cache = [torch.randn(1, 4, 16, 8) for _ in range(4)]
    out = w(ids, *cache)
    ref = cm(ids, past_kv=[(cache[0], cache[1]), (cache[2], cache[3])], use_cache=True)
    assert torch.allclose(out[0], ref[0]) and len(out) == 5
    assert io_names(2)[0] == ["input_ids", "k_lat_0", "v_lat_0", "k_lat_1", "v_lat_1"]
    # spec family (GQA): one step equals forward_cached
    cfg, m = _tiny()
    kv = KVCache(cfg, 1, 32, "cpu")
    prompt = torch.tensor([[1, 2, 3]])
    m.forward_cached(prompt, kv, prefill=True)
    want = m.forward_cached(torch.tensor([[7]]), kv)
    kv2 = KVCache(cfg, 1, 32, "cpu")
    m.forward_cached(prompt, kv2, prefill=True)
    flat = [t for l in range(cfg.n_layers) for t in (kv2.k[l], kv2.v[l])]
    got = DecodeStepWrapper(m)(torch.tensor([[7]]), torch.tensor(3), *flat)
    assert torch.allclose(got[0], want, atol=1e-4)


def test_decode_runner_matches_generate():
    import numpy as np
    from omnicoder.inference.generate import generate
    from omnicoder.inference.runtimes import DecodeRunner, TorchStepSession, bench_decode
    cfg, m = _tiny()
    prompt = torch.tensor([[4, 9, 17, 3]])
    want = generate(m, prompt, 6, temperature=0.0)
    sess = TorchStepSession(m, max_len=32)
    got = DecodeRunner(sess).generate(prompt.numpy(), 6)
    assert np.array_equal(got, want.numpy())
    q = DecodeRunner(sess, kv_quant="u8", group=16).generate(prompt.numpy(), 6)
    assert q.shape == got.shape and (q[:, :5] == got[:, :5]).all()
    assert bench_decode(sess, cfg.vocab_size, prompt_len=3, gen_tokens=3) > 0


def test_decode_runner_compat_window_and_sampling():
    import numpy as np
    from omnicoder.inference.runtimes import DecodeRunner, TorchStepSession, cache_layout
    from omnicoder.models.compat import OmniTransformer
    torch.manual_seed(0)
    cm = OmniTransformer(vocab_size=100, n_layers=2, d_model=32, n_heads=4, mlp_dim=64, n_experts=2, top_k=1,
                         max_seq_len=64, kv_latent_dim=8).eval()
    sess = TorchStepSession(cm)
    tok, pos, layers, outs = cache_layout(sess)
    assert tok == "input_ids" and pos is None and layers[0][2] == (1, 4, 16, 8) and outs[0] == "logits"
    r = DecodeRunner(sess, logit_bias={7: 1e4})
    out = r.generate(np.array([[1, 2, 3]]), 4, temperature=0.7, top_k=5, top_p=0.9, seed=1)
    assert out.shape == (1, 7) and (out[0, 3:] == 7).all()         # the bias dominates sampling


def test_lru_kv_pager_counts():
    from omnicoder.inference.runtimes import LRUKVPager, PagingConfig
    p = LRUKVPager(PagingConfig(n_layers=2, page_len=4, max_pages_ram=4, prefetch_ahead=1))
    for pos in range(16):
        p.access(pos)
    s = p.stats()
    assert s["misses"] == 2 and s["hits"] == 30 and s["prefetch_hits"] == 6 and s["resident_pages"] == 4
    small = LRUKVPager(PagingConfig(n_layers=2, page_len=4, max_pages_ram=2, prefetch_ahead=1))
    for pos in range(8):
        small.access(pos)
    assert small.stats()["misses"] > 2                              # prefetches evict the pages in use


def test_onnx_session_needs_onnxruntime():
    from omnicoder.inference import runtimes
    if runtimes.providers():
        pytest.skip("onnxruntime is installed")
    with pytest.raises(RuntimeError, match="onnxruntime"):
        runtimes.open_session("missing.onnx")


def test_logit_processor_penalties_and_bias():
    from omnicoder.inference.generate import LogitProcessor, generate, load_logit_bias
    p = LogitProcessor(1, 6, "cpu", repetition_penalty=2.0, presence_penalty=0.5, frequency_penalty=0.25,
                       logit_bias={5: 3.0})
    p.observe(torch.tensor([[1, 1, 2]]))
    x = p(torch.tensor([[1.0, 4.0, -2.0, 1.0, 0.0, 0.0]]))
    want = torch.tensor([[1.0, 4.0 / 2 - 0.5 - 0.5, -2.0 * 2 - 0.5 - 0.25, 1.0, 0.0, 3.0]])
    torch.testing.assert_close(x, want)
    assert not LogitProcessor(1, 6, "cpu").active
    cfg, m = _tiny()
    prompt = torch.tensor([[3, 4, 5]])
    out = generate(m, prompt, 12, temperature=0.0, repetition_penalty=1e6, presence_penalty=1e6)
    new = out[0, 3:].tolist()
    assert len(set(new)) == len(new) and not set(new) & {3, 4, 5}      # nothing repeats
    forced = generate(m, prompt, 5, temperature=0.0, logit_bias={42: 1e4})
    assert (forced[0, 3:] == 42).all()


def test_logit_processor_window_and_validation():
    """Only the last `window` tokens are penalised (the reference's rep_window); ids outside
    the vocabulary and a non-positive repetition penalty are refused."""
    from omnicoder.inference.generate import LogitProcessor
    p = LogitProcessor(2, 8, "cpu", frequency_penalty=1.0, window=3)
    p.observe(torch.tensor([[1, 2, 3, 4, 4], [5, 5, 5, 6, 7]]))      # longer than the window
    want = torch.zeros(2, 8)
    want[0, 3], want[0, 4] = 1, 2
    want[1, 5], want[1, 6], want[1, 7] = 1, 1, 1
    torch.testing.assert_close(p.counts, want)
    p.observe(torch.tensor([1, 7]))                                   # one step: the oldest leaves
    want[0, 3], want[0, 1] = 0, 1
    want[1, 5], want[1, 7] = 0, 2
    torch.testing.assert_close(p.counts, want)
    q = LogitProcessor(1, 8, "cpu", frequency_penalty=1.0, window=4)
    for t in [1, 2, 1, 3, 1, 4, 5, 6]:
        q.observe(torch.tensor([t]))
    assert q.counts[0].tolist() == [0, 1, 0, 0, 1, 1, 1, 0]            # the last four: 1, 4, 5, 6
    full = LogitProcessor(1, 8, "cpu", frequency_penalty=1.0, window=0)
    full.observe(torch.tensor([[1, 1, 1, 2]]))
    assert full.counts[0, 1] == 3
    with pytest.raises(ValueError):
        LogitProcessor(1, 8, "cpu", logit_bias={-1: 1.0})
    with pytest.raises(ValueError):
        LogitProcessor(1, 8, "cpu", logit_bias={8: 1.0})
    with pytest.raises(ValueError):
        LogitProcessor(1, 8, "cpu", repetition_penalty=0.0)


def test_generate_rejects_unknown_options():
    from omnicoder.inference.generate import generate
    cfg, m = _tiny()
    with pytest.raises(TypeError):
        generate(m, torch.tensor([[3, 4, 5]]), 2, temperature=0.0, no_such_option=True)


def test_load_logit_bias(tmp_path):
    from omnicoder.inference.generate import load_logit_bias
    f = tmp_path / "bias.json"
    f.write_text(json.dumps({"7": -5, "9": 2.5}))
    assert load_logit_bias(str(f)) == {7: -5.0, 9: 2.5}


# ---- decode-time add-ons of generate() ----------------------------------------------------
def test_addon_knn_blend_formula_and_generate():
    from omnicoder.inference.addons import DecodeAddons
    from omnicoder.inference.generate import generate
    from omnicoder.inference.knn_cache import KNNCache
    cfg, m = _tiny()
    kc = KNNCache(cfg.d_model, k=4)
    key = torch.randn(1, cfg.d_model)
    kc.add(key, torch.tensor([42]))
    ad = DecodeAddons(knn_cache=kc, knn_lambda=0.5, knn_write_every=0)
    logits = torch.randn(1, cfg.vocab_size)
    got = ad.apply(m, logits, key + 0.01)
    want = torch.log(0.5 * torch.softmax(logits, -1) + 0.5 * torch.nn.functional.one_hot(
        torch.tensor([42]), cfg.vocab_size).float())
    torch.testing.assert_close(got, want.clamp_min(torch.log(torch.tensor(1e-8))), rtol=1e-5, atol=1e-5)
    # through generate(): a near-certain kNN distribution forces its token; writes fill the cache
    kc2 = KNNCache(cfg.d_model, k=1)
    kc2.add(torch.zeros(1, cfg.d_model), torch.tensor([7]))
    out = generate(m, torch.tensor([[3, 4, 5]]), 6, temperature=0.0, knn_cache=kc2, knn_lambda=0.999,
                   knn_write_every=0)
    assert (out[0, 3:] == 7).all()
    kc3 = KNNCache(cfg.d_model)
    generate(m, torch.tensor([[3, 4, 5]]), 10, temperature=0.0, knn_cache=kc3, knn_lambda=0.2, knn_write_every=4)
    assert len(kc3) == 3                              # steps 0, 4, 8 of 10 (prefill + 9 decode steps)


def test_addon_retrieval_bias_matches_definition():
    from omnicoder.inference.addons import DecodeAddons, retrieval_vectors
    from omnicoder.inference.generate import generate
    cfg, m = _tiny()
    enc = lambda t: [ord(c) % cfg.vocab_size for c in t]
    r = retrieval_vectors(m, ["abc", "hello world"], enc)
    assert r.shape == (2, cfg.d_model)
    torch.testing.assert_close(r[0], m.embed[torch.tensor(enc("abc"))].mean(0))
    h = torch.randn(2, cfg.d_model)
    logits = torch.randn(2, cfg.vocab_size)
    got = DecodeAddons(retrieval_vecs=r, retrieval_alpha=0.7).apply(m, logits, h)
    w = torch.softmax(h @ r.t() / cfg.d_model ** 0.5, -1)
    torch.testing.assert_close(got, logits + 0.7 * ((w @ r) @ m.head_weight.t()), rtol=1e-5, atol=1e-5)
    out = generate(m, torch.tensor([[3, 4, 5]]), 4, temperature=0.0, retrieved_texts=["abc"],
                   retrieval_bias_alpha=0.5, encode_fn=enc)
    assert out.shape == (1, 7)
    with pytest.raises(ValueError):
        generate(m, torch.tensor([[3, 4, 5]]), 2, retrieved_texts=["abc"], retrieval_bias_alpha=0.5)


def test_addon_sfb_bias_prefers_goal_tokens():
    from omnicoder.inference.addons import sfb_token_bias
    from omnicoder.inference.generate import generate
    cfg, m = _tiny()
    enc = lambda t: [ord(c) % cfg.vocab_size for c in t]
    b = sfb_token_bias("1. compute xyz\n2. write code qq", enc, cfg.vocab_size, "cpu")
    goal_tok = set(enc("compute xyz") + enc("write code qq") + enc("1") + enc("2"))   # sub-goals and entities
    inside = b[torch.tensor(sorted(goal_tok))].min()
    outside = b[torch.tensor([t for t in range(cfg.vocab_size) if t not in goal_tok])].max()
    assert inside > outside
    out = generate(m, torch.tensor([[3, 4, 5]]), 4, temperature=0.0, sfb=True, sfb_alpha=50.0,
                   prompt_text="zzzz", encode_fn=enc)
    assert set(out[0, 3:].tolist()) <= {ord("z") % cfg.vocab_size}


def test_addon_adaptive_moe_top_k():
    from omnicoder.inference.addons import adapt_moe_top_k, clear_moe_top_k
    from omnicoder.inference.generate import generate
    cfg, m = _tiny()
    flat = torch.zeros(1, cfg.vocab_size)                       # uniform: not confident
    assert adapt_moe_top_k(m, flat, 1, 3, 0.3) == 3
    assert all(b.ffn.top_k_override == 3 for b in m.blocks)
    peaked = torch.full((1, cfg.vocab_size), -1e4)
    peaked[0, 5] = 0.0
    assert adapt_moe_top_k(m, peaked, 1, 3, 0.3, layer_ramp=True) == 1
    clear_moe_top_k(m)
    assert all(b.ffn.top_k_override is None for b in m.blocks)
    out = generate(m, torch.tensor([[3, 4, 5]]), 5, temperature=0.0, adaptive_moe=True, adaptive_top_k_min=1,
                   adaptive_top_k_max=3)
    assert out.shape == (1, 8) and all(b.ffn.top_k_override is None for b in m.blocks)


def test_prefix_embeds_equal_prepended_tokens():
    """Priming the cache with the embedding vectors of some tokens is the same as prepending them."""
    from omnicoder.inference.generate import generate
    cfg, m = _tiny()
    pre = torch.tensor([[11, 12, 13, 14]])
    prompt = torch.tensor([[3, 4, 5]])
    a = generate(m, torch.cat([pre, prompt], 1), 5, temperature=0.0)[:, pre.shape[1]:]
    b = generate(m, prompt, 5, temperature=0.0, prefix_embeds=m.embed[pre])
    assert torch.equal(a, b)


def test_speculative_verifier_threshold_and_early_exit():
    from omnicoder.inference.generate import generate
    cfg = ModelConfig(name="t", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=128,
                      verifier_head=True, attn=AttentionConfig(kind="gqa", n_kv_heads=2))
    tgt = build_model(cfg, device="cpu", seed=0).eval()
    dcfg = ModelConfig(name="d", vocab_size=300, d_model=32, n_layers=1, n_heads=2, ffn_dim=64, max_seq_len=128)
    drf = build_model(dcfg, device="cpu", seed=1).eval()
    prompt = torch.tensor([[3, 4, 5], [6, 7, 8]])
    plain = generate(tgt, prompt, 8, temperature=0.0)
    # an unreachable verifier threshold accepts nothing: every token comes from the target
    out, st = generate(tgt, prompt, 8, temperature=0.0, draft_model=drf, speculative_draft_len=3,
                       verify_threshold=1.5, return_stats=True)
    assert st.accepted_draft_tokens == 0 and torch.equal(out, plain)
    # a threshold every step meets: after the first step every step skips the draft
    out2, st2 = generate(tgt, prompt, 8, temperature=0.0, draft_model=drf, speculative_draft_len=3,
                         early_exit=True, early_exit_entropy=1e9, return_stats=True)
    assert torch.equal(out2, plain) and st2.early_exits == st2.steps - 1


def test_onnx_wrapper_mla_prefill_and_decode_match_model():
    """Spec MLA family through the export wrapper (absorbed latent attention): a T-token prefill
    graph and the following one-token decode steps give forward_cached's logits."""
    from omnicoder.export.onnx_export import DecodeStepWrapper, example_inputs, spec_cache_shapes
    cfg = ModelConfig(name="mla_x", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64,
                      attn=AttentionConfig(kind="mla", kv_lora_rank=32, qk_rope_dim=16, qk_nope_dim=16,
                                           v_head_dim=16),
                      moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=64, n_shared_experts=1))
    m = build_model(cfg, device="cpu", seed=0).eval()
    prompt = torch.tensor([[5, 9, 2, 7, 1, 3], [8, 8, 4, 6, 2, 11]])
    from omnicoder.inference.kv_cache import KVCache
    kv = KVCache(cfg, 2, 32, "cpu")
    want = [m.forward_cached(prompt, kv, prefill=True)]
    w = DecodeStepWrapper(m)
    cache = [torch.zeros(s) for s in spec_cache_shapes(cfg, 2, 32)]
    out = w(prompt, torch.tensor(0), *cache)
    torch.testing.assert_close(out[0], want[0], rtol=1e-4, atol=1e-4)
    cache = list(out[1:])
    pos = prompt.shape[1]
    for t in (4, 17, 23):
        ids = torch.tensor([[t], [t + 1]])
        ref = m.forward_cached(ids, kv)
        out = w(ids, torch.tensor(pos), *cache)
        torch.testing.assert_close(out[0], ref, rtol=1e-4, atol=1e-4)
        cache = list(out[1:])
        pos += 1
    w2, args = example_inputs(m, batch=1, max_len=16, tokens=4)
    assert args[0].shape == (1, 4) and len(args) == 2 + 2 * cfg.n_layers


def test_static_moe_and_runtime_exports(tmp_path):
    """The export-time routed experts (static shapes) equal the dropless torch path; the MoE decode
    step exports as a torch.export program that reproduces the wrapper; targets without their
    package are reported as skipped."""
    from omnicoder.config import get_preset
    from omnicoder.export.mobile_runtimes import export_all
    from omnicoder.export.onnx_export import example_inputs
    from omnicoder.ops.moe import moe_ffn_static, moe_ffn_torch
    g = torch.Generator().manual_seed(0)
    x, r = torch.randn(7, 64, generator=g), torch.randn(8, 64, generator=g)
    w13, w2 = torch.randn(8, 128, 64, generator=g) * 0.1, torch.randn(8, 64, 64, generator=g) * 0.1
    torch.testing.assert_close(moe_ffn_static(x, r, w13, w2, 2, True)[0], moe_ffn_torch(x, r, w13, w2, 2, 0, True)[0],
                               rtol=1e-5, atol=1e-5)
    m = build_model(get_preset("tiny_moe"), device="cpu", seed=0).eval()
    res = export_all(m, str(tmp_path), max_len=32)
    prog = torch.export.load(res["program"]["file"])
    w, args = example_inputs(m, 1, 32, 1)
    torch.testing.assert_close(prog.module()(*args)[0], w(*args)[0])
    assert "skipped" in res["executorch"] or "file" in res["executorch"]
    assert os.path.exists(res["mlc"]["recipe"])


def test_export_variants_bias_heads_multimodal_longctx(tmp_path):
    """Export variants: the logit_bias input shifts the logits; verifier / MTP head outputs equal
    the heads applied to the final hidden state; the multimodal prefill graph equals the model on
    the composer's embeddings; long-context copies interpolate RoPE; the sidecars are written; the
    variants trace under torch.export."""
    import json as _json

    from omnicoder.export.onnx_export import (DecodeStepWrapper, example_inputs, io_names, longctx_model,
                                              multimodal_example_inputs, spec_cache_shapes, write_sidecars)
    from omnicoder.multimodal.backbones import VisionBackbone
    from omnicoder.multimodal.composer import FusionComposer
    cfg = ModelConfig(name="exp_v", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64,
                      mtp_heads=2, verifier_head=True)
    m = build_model(cfg, device="cpu", seed=0).eval()
    ids = torch.tensor([[5, 9, 2], [8, 4, 6]])
    cache = [torch.zeros(s) for s in spec_cache_shapes(cfg, 2, 16)]
    base = DecodeStepWrapper(m)(ids, torch.tensor(0), *cache)
    bias = torch.zeros(2, 300)
    bias[:, 7] = 5.0
    wb = DecodeStepWrapper(m, logit_bias=True, heads=True)
    out = wb(ids, torch.tensor(0), *cache, bias)
    torch.testing.assert_close(out[0], base[0] + bias[:, None], rtol=1e-5, atol=1e-5)
    assert wb.head_names() == ["verifier_logits", "mtp_logits_0", "mtp_logits_1"]
    assert len(out) == 1 + 2 * cfg.n_layers + 3
    y = m.hidden(ids)[0].reshape(2, 3, -1)                   # final-norm hidden state of the plain forward
    torch.testing.assert_close(out[-3], y @ m.verifier.t(), rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(out[-1], y @ m.mtp_heads[1].t(), rtol=1e-4, atol=1e-4)
    ins, outs = io_names(cfg.n_layers, spec=True, logit_bias=True, head_names=wb.head_names())
    assert ins[-1] == "logit_bias" and outs[-1] == "mtp_logits_1"
    w, args = example_inputs(m, 1, 16, 1, logit_bias=True, heads=True)
    prog = torch.export.export(w, args, strict=False)
    torch.testing.assert_close(prog.module()(*args)[0], w(*args)[0])
    # multimodal prefill
    comp = FusionComposer(64, vision=VisionBackbone("vit_tiny", image_size=32, depth=1)).eval()
    mw, margs = multimodal_example_inputs(m, comp, image_size=32, text_tokens=4)
    got = mw(*margs)[0]
    emb, _ = comp.fuse_all(m.embed[margs[1]], image=margs[0])
    ref = m(None, embeds=emb, all_logits=True)["logits"]
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-4)
    # long context: positions interpolated by 32768 / 64
    lm = longctx_model(m, 32768)
    assert lm.cfg.attn.rope_scale == 32768 / 64 and lm.rope.max_pos == 32768 and m.cfg.attn.rope_scale == 1.0
    torch.testing.assert_close(lm.rope.cs[:, 512], m.rope.cs[:, 1])
    # sidecars
    paths = write_sidecars(m, str(tmp_path / "d.onnx"), 128, kv_page_len=32, kvq="nf4")
    meta = _json.load(open(paths[0]))
    assert meta["pages_per_layer"] == 4 and _json.load(open(paths[1]))["bits"] == 4


def test_generate_cli_retrieval_template_tools_certificate(tmp_path, capsys):
    """File retrieval picks the passage about the query; the CLI formats the prompt, runs tool calls
    in the output and emits a certificate; --target_ctx interpolates RoPE."""
    import json as _json

    from omnicoder.inference.generate import main, retrieve_passages
    from omnicoder.inference.tools import ToolRegistry
    (tmp_path / "a.txt").write_text("The capital of France is Paris. The Eiffel tower stands in Paris.\n" * 3)
    (tmp_path / "b.md").write_text("Python lists support append and pop; dictionaries map keys to values.\n" * 3)
    got = retrieve_passages(str(tmp_path), "where is the eiffel tower", k=1, chunk=120, stride=80)
    assert len(got) == 1 and "Eiffel" in got[0]
    assert ToolRegistry().run_calls("x <tool>calc(2*21)</tool>").endswith("<result>42</result>")
    main(["--preset", "tiny_moe", "--device", "cpu", "--max_new_tokens", "3", "--retrieve_path", str(tmp_path),
          "--retrieve_k", "1", "--retrieve_prepend", "--system_prompt", "S: ", "--tool_use", "--emit_cert",
          "--json", "--target_ctx", "16384", "--prompt", "where is the eiffel tower", "--no_cuda_graph"])
    out = _json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert "certificate" in out and out["stats"]["prompt_tokens"] > len("where is the eiffel tower")


def test_scmoe_contrast_decoding():
    """Self-contrast MoE: alpha 0 is plain decoding; a weak pass with as many experts as the strong
    one contrasts to the same distribution (greedy output unchanged); the first token follows
    (1 + a) log p_strong - a log p_weak computed by hand with top-1 routing."""
    from omnicoder.inference.generate import _prefill, generate
    from omnicoder.inference.kv_cache import KVCache
    torch.manual_seed(0)
    cfg = ModelConfig(name="sc", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64,
                      moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=64))
    m = build_model(cfg, device="cpu", seed=0).eval()
    ids = torch.tensor([[5, 9, 2, 7], [8, 1, 4, 6]])
    base = generate(m, ids, 5, temperature=0.0, top_k=0, top_p=1.0)
    assert torch.equal(generate(m, ids, 5, temperature=0.0, top_k=0, top_p=1.0, scmoe_alpha=0.0), base)
    assert torch.equal(generate(m, ids, 5, temperature=0.0, top_k=0, top_p=1.0, scmoe_alpha=0.7, scmoe_topk=2),
                       base)
    got = generate(m, ids, 1, temperature=0.0, top_k=0, top_p=1.0, scmoe_alpha=1.5, scmoe_topk=1)
    strong = _prefill(m, ids, KVCache(cfg, 2, 16, "cpu"))
    for b in m.blocks:
        b.ffn.top_k_override = 1
    weak = _prefill(m, ids, KVCache(cfg, 2, 16, "cpu"))
    for b in m.blocks:
        b.ffn.top_k_override = None
    want = (2.5 * torch.log_softmax(strong.float(), -1) - 1.5 * torch.log_softmax(weak.float(), -1)).argmax(-1)
    assert torch.equal(got[:, -1], want)
    assert all(b.ffn.top_k_override is None for b in m.blocks)      # restored after decoding
    with pytest.raises(ValueError):
        generate(m, ids, 2, scmoe_alpha=1.0, adaptive_moe=True)


def test_tool_fabric():
    from omnicoder.inference.tool_fabric import (analyze_inputs, combine_verifier_signals, invoke_tools_in_text,
                                                 media_paths)
    out = invoke_tools_in_text("sum: <tool>calc(2 + 3 * 4)</tool> done")
    assert "<result>14</result>" in out
    assert abs(combine_verifier_signals({"text": 1.0, "code": 0.0}, {"text": 3.0}) - 0.75) < 1e-9
    assert media_paths('look at "cat.png" and (talk.wav), not notes.txt') == ["cat.png", "talk.wav"]

    def detect(p):
        return ["cat", "sofa"]

    def transcribe(p):
        raise OSError("no such file")

    ctx, state, errors = analyze_inputs("is the cat.png on a sofa? listen: talk.wav clip.mp4", detect=detect,
                                        transcribe=transcribe)
    assert state.facts == ["cat present_in image cat.png", "sofa present_in image cat.png"]
    assert "FACT cat present_in image cat.png" in ctx
    assert len(errors) == 1 and "talk.wav" in errors[0] and "OSError" in errors[0]
    ctx, state, _ = analyze_inputs("cat.png", modes="audio", detect=detect)
    assert state.facts == [] and ctx == ""


def test_preference_expert_adapters_and_index(tmp_path):
    from omnicoder.config import ModelConfig
    from omnicoder.models.lm import build_model
    from omnicoder.training.preference_expert import (load_preference_lora, main, read_texts, token_windows,
                                                      train_preference_lora)
    from omnicoder.training.tokenizer import get_tokenizer
    d = tmp_path / "notes"
    d.mkdir()
    for i, t in enumerate(["I prefer tabs over spaces in Makefiles.", "My favourite language is Rust.",
                           "Always answer in British English, please."]):
        (d / f"n{i}.txt").write_text(t)
    texts = read_texts(str(d))
    assert len(texts) == 3
    cfg = ModelConfig(name="pe", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64)
    model = build_model(cfg, "cpu", dtype=torch.float32, seed=0)
    w = token_windows(texts, get_tokenizer(300), 16)
    assert w.shape[1] == 17
    base = {k: v.clone() for k, v in model.state_dict().items()}
    losses = train_preference_lora(model, w, steps=100, batch=4, lr=1e-2)
    assert sum(losses[-5:]) / 5 < 0.9 * losses[0]
    # only adapters trained: the frozen weights did not move
    sd = model.state_dict()
    assert all(torch.equal(sd[k], v) for k, v in base.items() if k in sd)
    out = tmp_path / "pref"
    assert main(["--data", str(d), "--preset", "tiny_moe", "--steps", "1", "--seq_len", "16", "--out_dir", str(out),
                 "--device", "cpu"]) == 0
    fresh = build_model(cfg.__class__.from_dict(__import__("omnicoder.config", fromlist=["get_preset"])
                                                .get_preset("tiny_moe").to_dict()), "cpu", dtype=torch.float32)
    assert load_preference_lora(fresh, str(out / "pref_lora.pt")) > 0
    from omnicoder.inference.generate import main as gen_main
    gen_main(["--preset", "tiny_moe", "--prompt", "which language", "--max_new_tokens", "2", "--device", "cpu",
              "--pref_lora", str(out / "pref_lora.pt"), "--pref_index", str(out / "index"), "--no_cuda_graph"])


def test_decode_runner_from_sidecars(tmp_path):
    import json

    import numpy as np
    from omnicoder.export.onnx_export import write_sidecars
    from omnicoder.inference.runtimes import DecodeRunner, TorchStepSession
    cfg, m = _tiny()
    path = str(tmp_path / "ds.onnx")
    write_sidecars(m, path, max_len=32, kv_page_len=8, kvq="u8", kvq_group=16)
    (tmp_path / "pf.json").write_text(json.dumps({"keep_pages": 1}))
    r = DecodeRunner.from_sidecars(TorchStepSession(m, max_len=32), path, str(tmp_path / "pf.json"))
    assert r.kv_quant == "u8" and r.group == 16 and r.pager.cfg.max_pages_ram == cfg.n_layers
    out = r.generate(np.array([[4, 9, 17, 3]]), 4)
    assert out.shape == (1, 8) and r.pager.stats()["hits"] + r.pager.stats()["misses"] > 0
    plain = DecodeRunner.from_sidecars(TorchStepSession(m, max_len=32), str(tmp_path / "none.onnx"))
    assert plain.kv_quant is None and plain.pager is None


def test_generate_cli_reference_flags(tmp_path, capsys):
    """The reference's generate flags that map onto this package: aliases, saved-index retrieval,
    multi-index search with a byte budget; FAISS-only flags fail with a clear message."""
    import json

    import pytest
    from omnicoder.inference.generate import main as gen_main
    from omnicoder.tools.utilities import main as tools_main
    for name, topic in (("a", "cuda kernels and tensor cores"), ("b", "python lists and loops")):
        d = tmp_path / "docs" / name
        d.mkdir(parents=True)
        for i in range(4):
            (d / f"{i}.txt").write_text(f"{topic} note number {i} " * 3)
        assert tools_main(["pq-build", str(d), str(tmp_path / "idx" / name), "--m", "2", "--ks", "2",
                           "--dim", "8"]) == 0
    base = ["--preset", "tiny_moe", "--prompt", "tensor cores", "--max_new_tokens", "1", "--device", "cpu",
            "--no_cuda_graph", "--json"]
    capsys.readouterr()
    gen_main(base + ["--multi_index_root", str(tmp_path / "idx"), "--mi_topk", "3", "--adaptive_gating",
                     "--retrieve_pq_index", str(tmp_path / "idx" / "a"), "--retrieve_k", "2"])
    got = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert got["retrieved_passages"] == 5
    gen_main(base + ["--multi_index_root", str(tmp_path / "idx"), "--retrieve_budget_bytes", "300"])
    got = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert got["retrieved_passages"] == 2                              # two 132-byte passages fit in 300
    with pytest.raises(SystemExit):
        gen_main(base + ["--retrieve_faiss", "x"])


def test_mtp_self_speculative_decoding_is_exact():
    """Drafts from the MTP heads, verified by the model itself: greedy output equals plain greedy decoding
    for prompts of one and several tokens; sampled decoding runs and counts its proposals."""
    from omnicoder.config import ModelConfig
    from omnicoder.inference.generate import generate
    from omnicoder.models.lm import build_model
    cfg = ModelConfig(name="mtp", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=128,
                      mtp_heads=3)
    m = build_model(cfg, "cpu", dtype=torch.float32, seed=0).eval()
    for prompt in (torch.tensor([[5]]), torch.tensor([[4, 9, 17, 3], [7, 7, 8, 1]])):
        want = generate(m, prompt, 12, temperature=0.0)
        got, st = generate(m, prompt, 12, temperature=0.0, speculative_draft_len=3, mtp_draft=True, return_stats=True)
        assert torch.equal(got, want) and st.proposed_draft_tokens > 0
    out, st = generate(m, torch.tensor([[4, 9, 17, 3]]), 8, temperature=0.9, speculative_draft_len=2,
                       mtp_draft=True, return_stats=True, seed=1)
    assert out.shape == (1, 12) and st.proposed_draft_tokens >= 2
    from omnicoder.inference.generate import main as gen_main
    gen_main(["--preset", "tiny_moe", "--prompt", "hi", "--max_new_tokens", "3", "--device", "cpu",
              "--no_cuda_graph", "--multi_token_heads", "3"])


def test_generate_cli_tree_reasoner(capsys):
    import json
    from omnicoder.inference.generate import main as gen_main
    capsys.readouterr()
    gen_main(["--preset", "tiny_moe", "--prompt", "2 + 2 =", "--max_new_tokens", "4", "--device", "cpu",
              "--no_cuda_graph", "--json", "--reasoner", "tot", "--tree_depth", "2", "--tree_width", "2",
              "--tree_iterations", "4"])
    got = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert "text" in got
    gen_main(["--preset", "tiny_moe", "--prompt", "hello", "--max_new_tokens", "2", "--device", "cpu",
              "--no_cuda_graph", "--json", "--reasoner", "omega"])
    got = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert "certificate" in got
