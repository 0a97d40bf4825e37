"""CPU tests of the multimodal VQ-VAEs and aligners, the multimodal / verifier trainers,
data mixtures, inference tools and retrieval memory, graph-of-thoughts and SFB
reasoning, GPTQ / AWQ quantisation, the mobile package round trip, tensor helpers
and checkpoint sidecars."""
import json
import os

import pytest
import torch
import torch.nn.functional as F


def _tiny_lm(vocab=64):
    from omnicoder.config import AttentionConfig, ModelConfig
    from omnicoder.models.lm import build_model
    return build_model(ModelConfig(vocab_size=vocab, d_model=32, n_layers=1, n_heads=4, ffn_dim=64, max_seq_len=64,
                                   attn=AttentionConfig(kind="mha")), seed=0)


# ---------------------------------------------------------------------------- multimodal
def test_image_vqvae_codes_and_training_reduce_loss():
    from omnicoder.multimodal.vqvae import ImageVQVAE
    from omnicoder.training.multimodal import train_vq
    torch.manual_seed(0)
    m = ImageVQVAE(width=16, levels=2, code_dim=8, codebook_size=32)
    img = torch.rand(2, 3, 16, 16) * 2 - 1
    codes = m.encode(img)
    assert codes.shape == (2, 4, 4) and codes.dtype == torch.long and int(codes.max()) < 32
    assert m.decode(codes).shape == img.shape
    losses = train_vq(m, iter(lambda: img, None), steps=30, lr=3e-3)
    assert losses[-1] < losses[0]


def test_video_and_audio_vq_shapes():
    from omnicoder.multimodal.vqvae import AudioVQ, MelVocoder, VideoVQVAE
    torch.manual_seed(0)
    v = VideoVQVAE(width=16, levels=2, code_dim=8, codebook_size=16)
    vid = torch.rand(1, 3, 3, 16, 16)
    rec, codes, loss = v(vid)
    assert rec.shape == vid.shape and codes.shape == (1, 3, 4, 4) and loss.dim() == 0
    assert v.decode(codes).shape == vid.shape
    a = AudioVQ(n_mels=16, dim=32, code_dim=8, codebook_size=16)
    wav = torch.randn(2, 4000)
    c = a.encode(wav)
    assert c.dim() == 2 and c.shape[0] == 2 and int(c.max()) < 16
    voc = MelVocoder(n_mels=16, width=32, ups=(4, 2))
    assert voc(torch.randn(2, 10, 16)).shape == (2, 10 * voc.hop)


def test_cross_modal_alignment_learns_pairing():
    from omnicoder.multimodal.aligner import CrossModalVerifier
    from omnicoder.training.multimodal import train_alignment
    torch.manual_seed(0)
    W = torch.randn(24, 16)

    def pairs():
        while True:
            t = torch.randn(8, 16)
            yield t, t @ W.t() + 0.01 * torch.randn(8, 24)
    ver = CrossModalVerifier({"text": 16, "image": 24}, shared=32)
    losses = train_alignment(ver, pairs(), steps=60, lr=1e-2)
    assert losses[-1] < 0.5 * losses[0]
    t, i = next(pairs())
    s = torch.stack([ver.score("text", t[k:k + 1].expand(8, -1), "image", i) for k in range(8)])
    assert (s.argmax(1) == torch.arange(8)).float().mean() >= 0.75


def test_grounding_segmentation_and_av_offset():
    from omnicoder.multimodal.aligner import GroundingHead, SegmentationHead, av_offset
    g = GroundingHead(32)
    box = g(torch.randn(2, 5, 32), torch.randn(2, 16, 32))
    assert box.shape == (2, 4) and bool(((box >= 0) & (box <= 1)).all())
    seg = SegmentationHead(32, n_classes=3)(torch.randn(2, 16, 32), grid=4, image_size=32)
    assert seg.shape == (2, 3, 32, 32)
    torch.manual_seed(0)
    video = torch.randn(40, 8)
    audio = torch.roll(video, shifts=-3, dims=0)          # audio frame t matches video frame t + 3
    assert av_offset(audio, video, max_lag=6) == 3


def test_vl_pretrain_step_and_verifier_head():
    from omnicoder.multimodal.composer import MultimodalComposer
    from omnicoder.multimodal.vocab import VocabSidecar
    from omnicoder.training.multimodal import VerifierHead, train_verifier_head, vl_pretrain_step
    lm = _tiny_lm(vocab=64)
    comp = MultimodalComposer(32, layout=VocabSidecar([0, 31], [32, 47], [48, 55], [56, 63]))
    opt = torch.optim.AdamW(lm.parameters(), lr=1e-3)
    loss = vl_pretrain_step(lm, comp, opt, torch.randint(0, 16, (2, 2, 2)), torch.randint(0, 32, (2, 9)))
    assert loss > 0
    head = VerifierHead(32)
    g = torch.Generator().manual_seed(0)

    def batches():
        while True:
            ids = torch.randint(0, 32, (8, 6), generator=g)
            yield ids, (ids[:, -1] < 16).long()
    ls = train_verifier_head(lm, head, batches(), steps=40, lr=1e-2)
    assert sum(ls[-5:]) < sum(ls[:5])


# ---------------------------------------------------------------------------- data
def test_data_module_noise_and_mixture(tmp_path):
    from omnicoder.training.data import DataEngine, DataModule, JsonlPairs, SyntheticTokens, TokenStream
    src = TokenStream(torch.arange(1, 2001) % 97 + 1, seq_len=16)
    dm = DataModule(src, batch=4, vocab=97, drop_p=0.5, seed=0)
    ids, lab = next(dm)
    assert ids.shape == (4, 16) and (ids == 0).float().mean() > 0.3 and (lab != 0).all()
    p = tmp_path / "pairs.jsonl"
    p.write_text("\n".join(json.dumps({"prompt": "ab", "response": "cde"}) for _ in range(3)))
    ds = JsonlPairs(str(p), lambda s: [ord(c) for c in s], seq_len=8)
    x, y = ds[0]
    assert x.tolist()[:5] == [97, 98, 99, 100, 101] and y.tolist()[:4] == [-100, 99, 100, 101]
    eng = DataEngine({"a": iter(int, 1), "b": iter(int, 1)}, {"a": 3.0, "b": 1.0}, seed=0)
    for _ in range(400):
        next(eng)
    assert 250 < eng.counts["a"] < 350


# ---------------------------------------------------------------------------- inference tools
def test_tool_registry_and_router():
    from omnicoder.inference.tools import ToolRegistry, UnifiedRouter, safe_eval_arith
    assert safe_eval_arith("2*(3+4)**2 - 1") == 97
    with pytest.raises(ValueError):
        safe_eval_arith("__import__('os')")
    reg = ToolRegistry()
    reg.register("upper", str.upper)
    out = reg.run_calls("x <tool>calc(6*7)</tool> y <tool>upper('hi')</tool> <tool>nope(1)</tool>")
    assert "<result>42</result>" in out and "<result>HI</result>" in out and "unknown tool" in out
    r = UnifiedRouter()
    r.register("text", lambda q: "T")
    r.register("image", lambda q: "I")
    assert r({"prompt": "x"}) == "T" and r({"path": "cat.PNG"}) == "I"
    with pytest.raises(KeyError):
        r({"modality": "audio"})


def test_estimate_memory_counts_parameters():
    from omnicoder.inference.tools import estimate_memory
    lm = _tiny_lm(vocab=64)
    est = estimate_memory(lm.cfg, batch=2, seq=128, kv_dtype="int8", training=True)
    n = sum(p.numel() for p in lm.parameters())
    assert abs(est["params"] - n) / n < 0.05, (est["params"], n)
    assert est["kv_cache_bytes"] > 0 and est["total_bytes"] > est["weights_bytes"]


def test_retrieval_and_semantic_memory():
    from omnicoder.inference.retrieval_memory import ExternalRetrievalMemory, SemanticMemory, retrieval_prefix
    mem = ExternalRetrievalMemory()
    mem.add(["the capital of France is Paris", "python lists have append", "rust uses ownership"])
    assert "Paris" in mem.search("what is the capital of France", k=1)[0][0]
    ids = retrieval_prefix(mem, "python append", lambda s: [len(w) for w in s.split()], k=1, sep=[0])
    assert ids[-1] == 0 and len(ids) == 5
    sm = SemanticMemory(half_life=2.0)
    sm.put("a", 1)
    for i in range(10):
        sm.put(f"x{i}", i)
    assert sm.relevance("a") < 0.1
    assert sm.get("x9") == 9 and sm.top(1) == ["x9"]
    assert sm.forget(0.05) >= 1 and "a" not in sm.facts


# ---------------------------------------------------------------------------- reasoning
def test_graph_of_thoughts_and_bfs():
    from omnicoder.reasoning.graph_of_thoughts import AdaptiveGraphOfThoughts, latent_bfs, reflect
    target = 23
    got = AdaptiveGraphOfThoughts(propose=lambda s: [s + 1, s * 2, s + 5], score=lambda s: -abs(target - s),
                                  is_final=lambda s: s == target, beam=3, max_rounds=10)
    assert got.run(1).state == target
    path = latent_bfs(1, lambda s: [("+1", s + 1), ("*2", s * 2)] if s < 100 else [], lambda s: s == 10)
    assert path is not None and len(path) == 4             # 1 -> 2 -> 4 -> 5 -> 10
    ans, rounds = reflect(lambda p: "ok" if "feedback" in p else "bad",
                          lambda p, a: (a == "ok", "try again"), "q")
    assert ans == "ok" and rounds == 1


def test_omega_controller_hysteresis():
    from omnicoder.reasoning.graph_of_thoughts import OmegaController
    oc = OmegaController()
    flat, sharp = torch.full((1, 100), 0.01), torch.nn.functional.one_hot(torch.tensor([3]), 100).float()
    assert oc.knobs(flat)["search"] and oc.mode == "explore"
    mid = torch.softmax(torch.randn(1, 100) * 2.0, -1)
    if oc.normalized_entropy(mid) > oc.low:
        assert oc.knobs(mid)["search"]                     # hysteresis: stays exploring
    assert not oc.knobs(sharp)["search"] and oc.mode == "normal"


def test_certificates():
    from omnicoder.reasoning.graph_of_thoughts import verify_certificate
    assert verify_certificate("42", {"kind": "numeric", "value": 42})
    assert not verify_certificate("41", {"kind": "numeric", "value": 42})
    assert verify_certificate(12, {"kind": "python", "check": "assert answer % 3 == 0"})
    assert not verify_certificate(13, {"kind": "python", "check": "assert answer % 3 == 0"})


def test_sfb_factorize_spn_bias_arbiter():
    from omnicoder.reasoning.sfb import ProofMarginArbiter, compile_factor_graph, cross_bias, factorize
    fs = factorize("1. compute 3 + 4\n2. implement a python function\n3. who wrote Hamlet?")
    assert [f["kind"] for f in fs] == ["math", "code", "retrieval"]
    spn = compile_factor_graph({"a": [0, 1], "b": [0, 1]},
                               [(("a",), lambda a: 0.3 if a else 0.7), (("a", "b"), lambda a, b: 0.9 if a == b else 0.1)])
    m = spn.marginal("b", [0, 1])
    assert abs(m[1] - (0.3 * 0.9 + 0.7 * 0.1)) < 1e-9
    assert abs(spn.marginal("a", [0, 1], {"b": 1})[1] - 0.27 / 0.34) < 1e-9
    p1, p2 = torch.tensor([0.7, 0.1, 0.1, 0.1]), torch.tensor([0.1, 0.7, 0.1, 0.1])
    b = cross_bias([p1, p2], [3.0, 1.0])
    assert int(b.argmax()) == 0 and torch.allclose(torch.softmax(b, -1), 0.75 * p1 + 0.25 * p2, atol=1e-5)
    arb = ProofMarginArbiter(0.1)
    assert arb.choose([{"answer": "x", "score": 0.9}, {"answer": "y", "score": 0.85}]) is None
    assert arb.choose([{"answer": "x", "score": 0.5, "verified": True}, {"answer": "y", "score": 0.9}]) == "x"


# ---------------------------------------------------------------------------- export / quantisation
def test_gptq_beats_rtn_on_calibration_data():
    from omnicoder.export.quantize import gptq_quantize, rtn_quantize
    torch.manual_seed(0)
    W = torch.randn(64, 256)
    X = torch.randn(512, 256) @ torch.randn(256, 256) * 0.2       # correlated activations
    q, s, Wg = gptq_quantize(W, X, bits=4, group=128)
    _, _, Wr = rtn_quantize(W, bits=4, group=128)
    assert q.dtype == torch.int8 and int(q.abs().max()) <= 7 and s.shape == (64, 2)
    assert torch.allclose(Wg, (q.float().view(64, 2, 128) * s[..., None]).view(64, 256), atol=1e-5)
    eg = (X @ (W - Wg).t()).pow(2).mean()
    er = (X @ (W - Wr).t()).pow(2).mean()
    assert eg < 0.8 * er, (eg, er)


def test_awq_scales_do_not_hurt():
    from omnicoder.export.quantize import awq_scales, rtn_quantize
    torch.manual_seed(0)
    W = torch.randn(32, 128)
    X = torch.randn(256, 128) * torch.linspace(0.05, 5.0, 128)      # a few salient channels
    s, Ws = awq_scales(W, X, bits=4, group=64)
    _, _, Wq = rtn_quantize(Ws, 4, 64)
    _, _, Wr = rtn_quantize(W, 4, 64)
    ea = (X @ W.t() - (X / s) @ Wq.t()).pow(2).mean()
    er = (X @ (W - Wr).t()).pow(2).mean()
    assert ea <= er * 1.0001


def test_mobile_package_round_trip(tmp_path):
    from omnicoder.export.mobile_packager import load_package, package_model
    lm = _tiny_lm(vocab=64).eval()
    man = package_model(lm, str(tmp_path / "pkg"))
    assert "weights_int4.pt" in man["files"] and "vocab.json" in man["files"]
    m2 = load_package(str(tmp_path / "pkg")).eval()
    ids = torch.randint(0, 64, (1, 12))
    with torch.no_grad():
        a = lm(ids, all_logits=True)["logits"].float()
        b = m2(ids, all_logits=True)["logits"].float()
    assert (a - b).abs().max() < 0.25 * a.abs().max()
    (tmp_path / "pkg" / "config.json").write_text("{}")
    with pytest.raises(ValueError):
        load_package(str(tmp_path / "pkg"))


# ---------------------------------------------------------------------------- utilities
def test_torchutils(tmp_path):
    from omnicoder.utils.torchutils import (guard_shape, safe_concat, safe_copy_into, safe_make_contiguous,
                                            safe_new_like, safe_torch_save)
    t = torch.ones(2, 3)
    assert safe_new_like(t, fill=2.0).sum() == 12
    with pytest.raises(ValueError):
        safe_copy_into(torch.zeros(3), t)
    assert safe_concat([t, None, torch.zeros(0, 3), t.double()]).dtype == torch.float64
    assert safe_make_contiguous(t.t()).is_contiguous()
    guard_shape(t, (2, None))
    with pytest.raises(ValueError):
        guard_shape(t, (3, None), "x")
    p = str(tmp_path / "a" / "x.pt")
    safe_torch_save({"t": t}, p)
    assert torch.equal(torch.load(p)["t"], t) and os.listdir(tmp_path / "a") == ["x.pt"]


def test_checkpoint_sidecar_manifest_registry(tmp_path):
    from omnicoder.multimodal.vocab import VocabSidecar
    from omnicoder.training.checkpoint import BestWeightsRegistry, save_with_sidecar, write_manifest
    lm = _tiny_lm()
    p = str(tmp_path / "m.pt")
    save_with_sidecar(p, lm, meta={"step": 7}, vocab=VocabSidecar.from_config(text_vocab=64))
    meta = json.load(open(p + ".meta.json"))
    assert meta["step"] == 7 and meta["params"] == sum(v.numel() for v in lm.state_dict().values())
    assert os.path.exists(p + ".vocab.json")
    assert "m.pt" in write_manifest(str(tmp_path))
    reg = BestWeightsRegistry(str(tmp_path / "best.json"))
    assert reg.register("code", "a.pt", 0.5) and not reg.register("code", "b.pt", 0.4)
    assert reg.register("code", "c.pt", 0.6)
    assert BestWeightsRegistry(str(tmp_path / "best.json")).best("code") == "c.pt"


# ---------------------------------------------------------------------------- preference / reward models
def test_reward_model_learns_preference():
    from omnicoder.training.preference import RewardModel, train_reward_model
    torch.manual_seed(0)
    rm = RewardModel(_tiny_lm(vocab=64))
    g = torch.Generator().manual_seed(0)

    def pairs():
        while True:
            base = torch.randint(3, 64, (8, 6), generator=g)
            yield torch.cat([base, torch.ones(8, 1, dtype=torch.long)], 1), torch.cat([base, torch.full((8, 1), 2)], 1)
    losses = train_reward_model(rm, pairs(), steps=60, lr=3e-3)
    assert sum(losses[-5:]) / 5 < 0.3 < losses[0]
    ch, rj = next(pairs())
    with torch.no_grad():
        assert (rm(ch) > rm(rj)).float().mean() == 1.0


def test_preference_trainer_moves_margin_and_keeps_reference_frozen():
    import copy
    from omnicoder.training.preference import PreferenceTrainer
    torch.manual_seed(0)
    pol = _tiny_lm(vocab=64)
    ref = copy.deepcopy(pol)
    ref_state = {k: v.clone() for k, v in ref.state_dict().items()}
    tr = PreferenceTrainer(pol, ref, lr=3e-3, beta=1.0, kl_coef=0.05)
    ch = torch.tensor([[5, 6, 7, 8, 9, 10]] * 4)
    rj = torch.tensor([[5, 6, 7, 11, 12, 13]] * 4)
    first = tr.step(ch, rj, prompt_len=3)
    for _ in range(15):
        last = tr.step(ch, rj, prompt_len=3)
    assert last["margin"] > first["margin"] + 0.5 and last["pref"] < first["pref"]
    assert all(torch.equal(v, ref.state_dict()[k]) for k, v in ref_state.items())


def test_idk_reward_shaping():
    from omnicoder.training.preference import reward_idk, wrote_idk
    assert wrote_idk("Honestly, I don't know.") and not wrote_idk("It is 4")
    assert reward_idk("the answer is 4", "4") == 1.0
    assert reward_idk("I am not sure, maybe 4", "4") == pytest.approx(1.2)
    assert reward_idk("I don't know", "4") == pytest.approx(-0.7)
    assert reward_idk("it is 5", "4") == pytest.approx(-1.5)


def test_mcts_selfplay_round_runs():
    from omnicoder.training.preference import MCTSSelfPlay, make_math_prompts
    torch.manual_seed(0)
    prompts = make_math_prompts(2, seed=1, max_operand=9)
    assert all(eval(p[:-1]) == t for p, t in prompts)
    chars = "0123456789+-*= "
    enc = lambda s: [chars.index(c) + 1 for c in s]
    dec = lambda ids: "".join(chars[i - 1] if 1 <= i <= len(chars) else "" for i in ids)
    sp = MCTSSelfPlay(_tiny_lm(vocab=32), enc, dec, branch=2, depth=2, iterations=6, max_new_tokens=3, group=2)
    stats = sp.round(prompts)
    assert set(stats) >= {"loss", "reward_mean", "search_reward_mean"}


def test_video_encoder_and_temporal_mixer():
    from omnicoder.multimodal.video import TemporalMixer, VideoEncoder
    torch.manual_seed(0)
    enc = VideoEncoder(image_size=32, patch=8, dim=32, depth=1, heads=2, temporal_kernel=3)
    feats, pooled = enc(torch.randn(2, 5, 3, 32, 32))
    assert feats.shape == (2, 5, 32) and pooled.shape == (2, 32)
    assert torch.allclose(pooled, feats.mean(1))
    mix = TemporalMixer(8, kernel_size=3)
    x = torch.randn(1, 9, 8)
    y0 = mix(x)
    x2 = x.clone()
    x2[:, 8] += 1.0                                   # a change at t=8 reaches only t=7, 8 (kernel 3)
    diff = (mix(x2) - y0).abs().amax(-1)[0]
    assert diff[:7].max() == 0 and diff[7:].min() > 0


def test_voxel_head_and_ortho_renderer():
    from omnicoder.multimodal.video import OrthoRenderer, VoxelLatentHead
    torch.manual_seed(0)
    vox = VoxelLatentHead(16, depth=4, height=8, width=8, hidden=32)(torch.randn(2, 7, 16))
    assert vox.shape == (2, 4, 8, 8)
    r = OrthoRenderer(depth=4, out_h=16, out_w=16)
    img = r(vox)
    assert img.shape == (2, 3, 16, 16) and img.min() >= 0 and img.max() <= 1
    # a fully opaque front slice shows only its own colour
    opaque = torch.full((1, 4, 16, 16), -30.0)
    opaque[:, 0] = 30.0
    out = r(opaque)
    assert torch.allclose(out[0, :, 8, 8], torch.sigmoid(r.color[0]), atol=1e-4)
    assert torch.allclose(r(torch.full((1, 4, 16, 16), -30.0)), torch.zeros(1, 3, 16, 16), atol=1e-6)


def test_latent_refiner_and_interpolator():
    from omnicoder.multimodal.video import LatentInterpolator, LatentRefiner
    torch.manual_seed(0)
    ref = LatentRefiner(16)
    with torch.no_grad():
        ref.gate.zero_()
    x = torch.randn(3, 16)
    assert torch.equal(ref(x), x)                     # gate 0 is the identity
    assert LatentRefiner(16, temporal=True)(torch.randn(2, 6, 16)).shape == (2, 6, 16)
    with pytest.raises(ValueError):
        ref(torch.randn(2, 2, 2, 16))
    interp = LatentInterpolator(8, hidden=32)
    z0, z1 = torch.randn(2, 3, 8), torch.randn(2, 3, 8)
    out = interp(z0, z1, steps=5)
    assert out.shape == (2, 5, 3, 8)
    opt = torch.optim.Adam(interp.parameters(), lr=1e-2)
    tau = torch.linspace(0, 1, 5).view(1, 5, 1, 1)
    target = z0.unsqueeze(1) * (1 - tau) + z1.unsqueeze(1) * tau
    first = float(F.mse_loss(interp(z0, z1, 5), target))
    for _ in range(200):
        loss = F.mse_loss(interp(z0, z1, 5), target)
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert float(loss) < 0.2 * first


def _mm_setup():
    from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig
    from omnicoder.models.lm import build_model
    from omnicoder.multimodal.vocab import VocabSidecar
    cfg = ModelConfig(name="mm", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=256,
                      attn=AttentionConfig(kind="gqa", n_kv_heads=2), moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=64))
    return build_model(cfg, device="cpu", seed=0).eval(), VocabSidecar([0, 99], [100, 163], [164, 227], [228, 291])


def test_generate_codes_in_range_and_greedy():
    from omnicoder.multimodal.generation import generate_codes
    m, _ = _mm_setup()
    prompt = torch.tensor([[5, 6, 7]])
    codes = generate_codes(m, prompt, 100, 64, 6, temperature=0.0)
    assert codes.shape == (1, 6) and codes.min() >= 0 and codes.max() < 64
    ids = prompt
    for c in codes[0].tolist():                          # greedy equals argmax over the range, step by step
        with torch.no_grad():
            logits = m(ids)["logits"][0, -1]
        assert int(logits[100:164].argmax()) == c
        ids = torch.cat([ids, torch.tensor([[100 + c]])], 1)
    with pytest.raises(ValueError):
        generate_codes(m, prompt, 280, 64, 2)


def test_http_image_and_video_endpoints():
    import base64
    from fastapi.testclient import TestClient
    from omnicoder.multimodal.vqvae import ImageVQVAE, VideoVQVAE
    from omnicoder.tools.http_server import create_app
    m, voc = _mm_setup()
    torch.manual_seed(0)
    iv = ImageVQVAE(width=8, levels=2, code_dim=8, codebook_size=64)
    vv = VideoVQVAE(width=8, levels=2, code_dim=8, codebook_size=64)
    with TestClient(create_app(m, image_vq=iv, video_vq=vv, vocab=voc)) as cli:
        r = cli.post("/generate/image", json={"prompt": "a cat", "grid_h": 3, "grid_w": 2, "seed": 1}).json()
        assert r["shape"] == [3, 12, 8] and len(base64.b64decode(r["pixels_b64"])) == 3 * 12 * 8
        v = cli.post("/generate/video", json={"prompt": "waves", "grid_h": 2, "grid_w": 2, "frames": 3,
                                              "temperature": 0.0}).json()
        assert v["shape"] == [3, 3, 8, 8] and v["layout"] == "TCHW"
    with TestClient(create_app(m)) as cli:
        assert cli.post("/generate/image", json={"prompt": "x"}).status_code == 501


def test_btm_merge_round_robin_and_mean():
    from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig
    from omnicoder.models.lm import build_model
    from omnicoder.training.multimodal_tasks import btm_merge
    cfg = ModelConfig(name="b", vocab_size=300, d_model=64, n_layers=1, n_heads=4, ffn_dim=128, max_seq_len=64,
                      attn=AttentionConfig(kind="gqa", n_kv_heads=2), moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=64))
    d0, d1, st = (build_model(cfg, device="cpu", seed=s) for s in (1, 2, 3))
    rep = btm_merge(st, [d0, d1])
    w, a, b = st.state_dict()["blocks.0.ffn.w13"], d0.state_dict()["blocks.0.ffn.w13"], d1.state_dict()["blocks.0.ffn.w13"]
    assert torch.equal(w[0], a[0]) and torch.equal(w[1], b[0]) and torch.equal(w[2], a[1]) and torch.equal(w[3], b[1])
    q = st.state_dict()["blocks.0.attn.wqkv"]
    torch.testing.assert_close(q.float(), (d0.state_dict()["blocks.0.attn.wqkv"].float()
                                            + d1.state_dict()["blocks.0.attn.wqkv"].float()) / 2)
    assert rep["blocks.0.ffn.w2"] == "experts round-robin" and rep["embed"] == "mean of 2"


def test_latent3d_video_sr_policy_trainers_reduce_loss():
    from omnicoder.multimodal.video import OrthoRenderer, TemporalMixer, VoxelLatentHead
    from omnicoder.training import multimodal_tasks as mt
    torch.manual_seed(0)
    m, _ = _mm_setup()
    ids = torch.randint(0, 100, (2, 8))
    target = torch.zeros(2, 3, 16, 16)
    target[:, 0, 4:12, 4:12] = 1.0
    l3 = mt.train_latent3d(m, VoxelLatentHead(64, depth=4, height=8, width=8, hidden=32),
                           OrthoRenderer(depth=4, out_h=16, out_w=16), iter(lambda: (ids, target), None), 60, lr=3e-2)
    assert l3[-1] < 0.5 * l3[0]
    mix = TemporalMixer(8, kernel_size=3, causal=True)
    x = torch.randn(1, 9, 8)
    x2 = x.clone()
    x2[:, 5] += 1.0
    assert torch.equal(mix(x)[:, :5], mix(x2)[:, :5])               # causal: the past ignores frame 5
    t = torch.arange(12).float()
    clip = torch.stack([torch.sin(0.5 * t + p) for p in range(8)], -1)[None]
    lv = mt.train_video_temporal(mix, iter(lambda: clip, None), 150, lr=1e-2, smoothness=0.01)
    assert lv[-1] < 0.3 * lv[0]
    hr = torch.rand(2, 3, 16, 16)
    lr_img = F.avg_pool2d(hr, 2)
    ls = mt.train_super_resolution(mt.SuperResolver(2, width=16, depth=2), iter(lambda: (lr_img, hr), None), 80,
                                   lr=3e-3)
    assert ls[-1] < ls[0]
    r = mt.retention_targets(10, 4)
    assert r[-4:].eq(1).all() and r[0] == 0 and bool((r[1:6] > r[:5]).all())
    lp = mt.train_policy_head(m, torch.nn.Linear(64, 1), iter(lambda: ids, None), 60, lr=3e-2,
                              target_fn=lambda i: mt.retention_targets(i.shape[1], 3).expand(i.shape))
    assert lp[-1] < lp[0]
    p, q = torch.randn(2, 3, 8, 8), torch.randn(2, 3, 8, 8)
    assert float(mt.recon_loss(p, q, "huber")) > 0 and float(mt.recon_loss(p, p, "mae")) == 0
    assert float(mt.recon_loss(p, q, "feature", features=torch.nn.Conv2d(3, 4, 3))) > 0


def test_vector_index_exact_ivf_and_text_retriever():
    from omnicoder.retrieval.vector_index import IVFIndex, TextRetriever, VectorIndex
    torch.manual_seed(0)
    x = torch.randn(1000, 32)
    q = torch.randn(5, 32)
    for metric in ("cosine", "ip", "l2"):
        idx = VectorIndex(32, metric, chunk=300)
        idx.add(x)
        s, i = idx.search(q, 4)
        if metric == "l2":
            want = torch.cdist(q, x).topk(4, largest=False).indices
        else:
            xx = F.normalize(x, dim=1) if metric == "cosine" else x
            qq = F.normalize(q, dim=1) if metric == "cosine" else q
            want = (qq @ xx.t()).topk(4).indices
        assert torch.equal(i, want), metric
    ivf = IVFIndex(32, n_lists=16, nprobe=16)                 # probing every list is exact
    ivf.add(x)
    _, ii = ivf.search(q, 4)
    assert torch.equal(ii, (F.normalize(q, dim=1) @ F.normalize(x, dim=1).t()).topk(4).indices)
    docs = ["the cat sat on the mat " * 3, "gpu kernels use tensor memory and tma loads " * 3,
            "rivers flow into the sea " * 3]
    tr = TextRetriever(docs, dim=512, chunk_words=16, stride=12)
    assert "tensor" in tr.search("tensor memory kernels", k=1)[0].text


def test_media_metrics():
    from omnicoder.eval import media_metrics as mm
    assert mm.word_error_rate("the cat sat", "the cat sat") == 0
    assert mm.word_error_rate("the cat sat down", "the bat sat") == pytest.approx(0.5)
    assert mm.bleu(["the cat is on the mat"], [["the cat is on the mat"]]) == pytest.approx(1.0)
    assert 0 < mm.bleu(["the cat is on a mat today"], [["the cat is on the mat"]]) < 1
    assert mm.exact_match_accuracy([("Paris.", "paris"), ("4", "5")]) == 0.5
    torch.manual_seed(0)
    a = torch.rand(2, 3, 32, 32)
    assert mm.psnr(a, a) == float("inf") and mm.ssim(a, a) == pytest.approx(1.0, abs=1e-5)
    noisy = (a + 0.1 * torch.randn_like(a)).clamp(0, 1)
    assert 15 < mm.psnr(noisy, a) < 30 and mm.ssim(noisy, a) < mm.ssim(a, a)
    f1, f2 = torch.randn(500, 8), torch.randn(500, 8) + 2.0
    assert mm.frechet_distance(f1, f1) == pytest.approx(0.0, abs=1e-6)
    assert mm.frechet_distance(f1, f2) == pytest.approx(32.0, rel=0.15)   # |mu diff|^2 = 8 * 4
    assert mm.embedding_alignment(f1, f1) == pytest.approx(1.0)
    assert mm.temporal_consistency(torch.ones(5, 4)) == pytest.approx(1.0)
    s = torch.randn(1000)
    assert mm.snr_db(s, s + 0.1 * torch.randn(1000)) == pytest.approx(20.0, abs=1.5)


def test_train_flops_per_token_by_hand():
    from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig
    from omnicoder.utils.flops import active_params_per_token, mfu, train_flops_per_token
    cfg = ModelConfig(name="f", vocab_size=100, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64,
                      attn=AttentionConfig(kind="gqa", n_kv_heads=2),
                      moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=32, n_shared_experts=1))
    attn = 64 * 16 * (4 + 2 * 2) + 4 * 16 * 64                 # wqkv + wo
    ffn = 3 * (3 * 64 * 32) + 4 * 64                           # 2 routed + 1 shared expert, router
    assert active_params_per_token(cfg) == 2 * (attn + ffn) + 100 * 64
    fpt = train_flops_per_token(cfg, 32)
    assert fpt == 6 * active_params_per_token(cfg) + 3 * 2 * 2 * 16 * 4 * (16 + 16)
    assert mfu(1e12 / fpt, cfg, 32, 1, 1.0) == pytest.approx(1.0)


def test_import_changes_no_torch_flags():
    import subprocess
    import sys
    code = ("import torch\n"
            "f = lambda: (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32,\n"
            "             torch.get_float32_matmul_precision(), torch.are_deterministic_algorithms_enabled())\n"
            "a = f()\n"
            "import omnicoder, omnicoder.ops, omnicoder.models.lm, omnicoder.training.engine, omnicoder.parallel.zero\n"
            "assert f() == a, (a, f())\n")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=120,
                       cwd=os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    assert r.returncode == 0, r.stderr[-500:]


def test_expert_load_diagnostic():
    from omnicoder.config import AttentionConfig, ModelConfig, MoEConfig
    from omnicoder.models.lm import build_model
    from omnicoder.utils.diagnostics import expert_load
    cfg = ModelConfig(name="d", vocab_size=200, d_model=64, n_layers=3, n_heads=4, ffn_dim=128, max_seq_len=64,
                      attn=AttentionConfig(kind="gqa", n_kv_heads=2), moe=MoEConfig(n_experts=4, top_k=2, ffn_dim=32))
    m = build_model(cfg, device="cpu", seed=0)
    ids = torch.randint(0, 200, (2, 16))
    r = expert_load(m, ids)
    assert r["counts"].shape == (3, 4) and (r["counts"].sum(1) == 2 * 16 * 2).all()
    assert len(r["cv"]) == 3 and all(0.25 <= s <= 1.0 for s in r["max_share"])
    assert not m.blocks[0].ffn._forward_pre_hooks                       # hooks removed
