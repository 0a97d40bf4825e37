"""Vision backbone family and the full fusion-composer contract (continuous fusion with segment
ids, code tokenisation into the unified vocabulary and back to pixels / waveforms, grounding and
segmentation heads, video change scores, audio-video offset, router conditioning) on CPU."""
import pytest
import torch

from omnicoder.multimodal import (AudioVQ, FusionComposer, ImageVQVAE, MelFrontend, MelVocoder, VisionBackbone)
from omnicoder.multimodal.video import VideoEncoder


@pytest.mark.parametrize("backend,n_tok", [("vit_tiny", 16), ("dino_tiny", 16), ("siglip_tiny", 16)])
def test_vision_backbones(backend, n_tok):
    vb = VisionBackbone(backend, image_size=64, patch=16, depth=2)
    tok, pooled = vb(torch.randn(2, 3, 64, 64))
    assert tok.shape == (2, n_tok, 192) and pooled.shape == (2, 192)
    with pytest.raises(ValueError):
        VisionBackbone("convnext_tiny")


def test_fusion_composer_contract():
    torch.manual_seed(0)
    D = 64
    fc = FusionComposer(D, vision=VisionBackbone("vit_tiny", image_size=64, patch=16, depth=1),
                        video=VideoEncoder(image_size=32, patch=16, dim=48, depth=1, heads=2),
                        audio=MelFrontend(out_dim=40), image_vq=ImageVQVAE(width=16, levels=2, codebook_size=256),
                        audio_vq=AudioVQ(dim=32, codebook_size=128), vocoder=MelVocoder(width=32))
    text = torch.randn(2, 5, D)
    img = torch.randn(2, 3, 64, 64)
    vid = torch.randn(2, 3, 3, 32, 32)
    wav = torch.randn(2, 1600)
    emb, seg = fc.fuse_all(text, image=img, video=vid, audio=wav)
    n_aud = fc.audio_tokens(wav).shape[1]
    assert emb.shape == (2, (16 + 2) + (3 + 2) + (n_aud + 2) + 5, D) and seg.shape == emb.shape[:2]
    assert seg[0, 0] == 1 and seg[0, 18] == 2 and seg[0, -1] == 0 and (seg == 3).sum() == 2 * (n_aud + 2)
    assert fc.fuse_text_image(text, img).shape[1] == 18 + 5
    # discrete path: codes into the unified vocabulary and back
    codes = fc.encode_image_to_codes(img)
    assert codes.shape == (2, 16 * 16)
    ids = fc.fuse_text_image_codes(torch.zeros(2, 3, dtype=torch.long), codes.view(2, 16, 16).flatten(1))
    lo = fc.layout.image_range[0]
    assert ids.shape == (2, 256 + 3) and int(ids[:, :256].min()) >= lo
    assert fc.decode_image_from_codes(codes, (16, 16)).shape == (2, 3, 64, 64)
    acodes = fc.encode_audio_to_codes(wav)
    wave = fc.decode_audio_from_codes(acodes)
    assert wave.dim() == 2 and wave.shape[0] == 2 and wave.abs().max() <= 1.0
    assert fc.audio_vq.reconstruction_loss(wav) > 0
    # heads
    out = fc.vision_heads(fc.image_tokens(img), text, image_size=64)
    assert out["box"].shape == (2, 4) and out["mask_logits"].shape == (2, 1, 64, 64)
    vh = fc.video_heads(fc.video_tokens(vid))
    assert vh["change"].shape == (2, 2) and vh["keyframe"].shape == (2,)
    a = torch.randn(2, 12, 40)
    v = torch.cat([torch.randn(2, 2, 48), torch.randn(2, 12, 48)], 1)
    assert len(fc.av_sync(a, v[:, :12])["offset"]) == 2
    cond = fc.conditioning_from_hidden(emb, seg)
    assert set(cond) == {"text", "image", "video", "audio"} and cond["image"].shape == (2, D)
    with pytest.raises(RuntimeError):
        FusionComposer(D).encode_video_to_codes(vid)


def test_vl_task_trainers(tmp_path):
    """VQA / captioning over composed image features: only target tokens are trained, the loss
    falls on a fixed batch, JSONL rows load tensor files; ASR over audio features."""
    import json

    from omnicoder.config import AttentionConfig, ModelConfig
    from omnicoder.models.lm import build_model
    from omnicoder.training.tokenizer import get_tokenizer
    from omnicoder.training.vl_tasks import VLTaskTrainer, read_task_jsonl
    torch.manual_seed(0)
    cfg = ModelConfig(name="vl", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=128,
                      attn=AttentionConfig(kind="gqa", n_kv_heads=2))
    lm = build_model(cfg, device="cpu", seed=0)
    tok = get_tokenizer(cfg.vocab_size)
    fc = FusionComposer(64, vision=VisionBackbone("vit_tiny", image_size=32, patch=16, depth=1),
                        audio=MelFrontend(out_dim=32))
    tr = VLTaskTrainer(lm, fc, tok, "vqa", lr=3e-3)
    imgs = torch.randn(2, 3, 32, 32)
    b = tr.build(imgs, ["Question: color? Answer:", "Question: count? Answer:"], ["red", "two"])
    n_pre = 4 + 2                                       # 4 patches + begin / end markers
    assert (b.labels[:, :n_pre + 5] == -100).all()      # modality and prompt positions are not trained
    assert (b.labels != -100).sum() == len(tok.encode(" red")) + len(tok.encode(" two")) + 2
    losses = [tr.step(imgs, ["Question: color? Answer:"] * 2, ["red", "two"]) for _ in range(15)]
    assert losses[-1] < 0.5 * losses[0]
    torch.save(torch.randn(3, 32, 32), tmp_path / "a.pt")
    (tmp_path / "cap.jsonl").write_text(json.dumps({"image": str(tmp_path / "a.pt"), "caption": "a cat"}))
    rows = read_task_jsonl(str(tmp_path / "cap.jsonl"), "caption")
    cap = VLTaskTrainer(lm, fc, tok, "caption", lr=1e-3)
    assert len(cap.fit(rows, steps=2, batch=2)) == 2 and isinstance(cap.answer(rows[0]["media"], "Caption:", 3), str)
    asr = VLTaskTrainer(lm, fc, tok, "asr", lr=1e-3)
    assert asr.step(torch.randn(2, 1600), ["Transcript:"] * 2, ["hi", "yo"]) > 0


def test_av_sync_grounding_segmentation_heads():
    from omnicoder.multimodal.heads import ASRAdapter, AVSyncModule, RepRTAHead, TextSegHead, TTSAdapter
    torch.manual_seed(0)
    av = AVSyncModule(d_audio=40, d_video=24, d_model=64, num_heads=4)
    vf, score = av(torch.randn(2, 12, 40), torch.randn(2, 9, 24))
    assert vf.shape == (2, 9, 64) and score.shape == (2, 1) and bool(((score >= 0) & (score <= 1)).all())
    score.sum().backward()                                         # the score trains the projections
    assert av.audio_proj.weight.grad is not None
    head = RepRTAHead(d_model=32, num_props=5)
    toks, text = torch.randn(2, 16, 32), torch.randn(2, 32)
    boxes, conf = head(toks, text)
    assert boxes.shape == (2, 5, 4) and conf.shape == (2, 5)
    assert bool(((boxes > 0) & (boxes < 1)).all())
    assert not torch.allclose(boxes[:, 0], boxes[:, 1])            # proposals differ
    b2, c2 = RepRTAHead(d_model=32, num_props=8)(torch.randn(1, 4, 32), torch.randn(1, 32))
    assert b2.shape == (1, 8, 4) and torch.isinf(c2[0, 4:]).all()  # fewer tokens than proposals
    mask = TextSegHead(d_model=32)(toks, text)
    assert mask.shape == (2, 1, 4, 4) and bool(((mask >= 0) & (mask <= 1)).all())
    assert TextSegHead(d_model=32, grid_hw=(3, 6))(toks).shape == (2, 1, 3, 6)
    for a in (ASRAdapter(), TTSAdapter()):
        assert isinstance(a.available(), bool)


def test_flow_recon_trainer_learns_latents(tmp_path):
    """Reconstruction and rectified-flow training of the latent head: both losses fall on a
    two-image task, and flow sampling from noise lands near the target latents."""
    from omnicoder.config import ModelConfig
    from omnicoder.models.lm import build_model
    from omnicoder.training.flow_recon import FlowReconTrainer, LatentQueryHead, PatchPoolEncoder, main
    torch.manual_seed(0)
    cfg = ModelConfig(name="fr", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64)
    lm = build_model(cfg, "cpu", dtype=torch.float32, seed=0).eval()
    enc = PatchPoolEncoder(grid=2, channels=8)
    imgs = torch.stack([torch.zeros(3, 16, 16), torch.ones(3, 16, 16)])
    imgs[0, 0] = 1.0
    ids = torch.tensor([[5, 6, 7], [8, 9, 10]])
    z0 = enc(imgs)
    for flow in (False, True):
        torch.manual_seed(1)
        head = LatentQueryHead(64, 4, 8, width=64)
        tr = FlowReconTrainer(lm, head, enc, lr=3e-3, flow=flow)
        losses = [tr.step(imgs, ids) for _ in range(300)]
        assert sum(losses[-20:]) < 0.3 * sum(losses[:20]), (flow, losses[:3], losses[-3:])
        z = tr.sample(ids, steps=32)
        err = (z - z0).norm() / z0.norm()
        assert err < (0.2 if not flow else 0.5), (flow, float(err))
    assert main(["--steps", "2", "--device", "cpu", "--out", str(tmp_path / "h.pt")]) == 0


def test_pre_align_infonce_aligns_text_and_media(tmp_path):
    from omnicoder.multimodal.encoders import MelFrontend
    from omnicoder.training.pre_align import PreAlignTrainer, TextEmbedder, main

    class Flat(torch.nn.Module):               # tiny image encoder: mean colour -> features
        dim = 32

        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Linear(3, 32)

        def forward(self, x):
            return self.lin(x.mean((2, 3)))

    torch.manual_seed(0)
    tr = PreAlignTrainer(TextEmbedder(64, 32), {"image": Flat(), "audio": MelFrontend(out_dim=32)}, shared=16,
                         lr=1e-2)
    colors = torch.rand(8, 3)
    ids = torch.arange(1, 9)[:, None].repeat(1, 3)
    imgs = colors[:, :, None, None].expand(-1, -1, 8, 8)
    t = torch.arange(2000) / 16000.0
    wav = torch.stack([torch.sin(2 * 3.14159 * (200 + 100 * i) * t) for i in range(8)])
    first = tr.step(ids, image=imgs, audio=wav)
    for _ in range(150):
        last = tr.step(ids, image=imgs, audio=wav)
    assert last["image"] < 0.5 * first["image"] and last["audio"] < first["audio"]
    assert main(["--steps", "1", "--batch", "4", "--device", "cpu", "--out", str(tmp_path / "p.pt")]) == 0


def test_audio_recon_trainer_learns_latents(tmp_path):
    """Audio latent reconstruction with the spectral side losses: the loss falls on distinct tones
    and the predicted latents approach the mel-pooled targets; the CLI runs one flow-mode step."""
    from omnicoder.config import ModelConfig
    from omnicoder.models.lm import build_model
    from omnicoder.training.audio_recon import AudioReconTrainer, MelPoolEncoder, main, synthetic_tones
    from omnicoder.training.flow_recon import LatentQueryHead
    torch.manual_seed(0)
    cfg = ModelConfig(name="ar", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64)
    lm = build_model(cfg, "cpu", dtype=torch.float32, seed=0).eval()
    enc = MelPoolEncoder(segments=2, channels=8)
    waves, _ = synthetic_tones(3, samples=4000)
    ids = torch.tensor([[5, 6, 7], [8, 9, 10], [11, 12, 13]])
    z0 = enc(waves)
    assert z0.shape == (3, 2, 8) and torch.equal(z0, MelPoolEncoder(segments=2, channels=8)(waves))
    head = LatentQueryHead(64, 2, 8, width=64)
    tr = AudioReconTrainer(lm, head, enc, lr=3e-3)
    losses = [tr.step(waves, ids) for _ in range(200)]
    assert sum(losses[-10:]) < 0.3 * sum(losses[:10]), (losses[:3], losses[-3:])
    err = (tr.sample(ids) - z0).norm() / z0.norm()
    assert err < 0.2, float(err)
    assert main(["--steps", "1", "--batch", "2", "--flow_loss", "--device", "cpu", "--out",
                 str(tmp_path / "a.pt")]) == 0


def test_concept_align_retrieves_own_image(tmp_path):
    """Concept-head alignment against a frozen pre-aligned teacher: InfoNCE + triplet terms fall and
    most captions' concept embeddings end closest to their own image (the random teacher's text and
    image embeddings of an item disagree, so the two InfoNCE terms pull against each other)."""
    from omnicoder.config import ModelConfig
    from omnicoder.models.heads import ConceptLatentHead
    from omnicoder.models.lm import build_model
    from omnicoder.multimodal.aligner import PreAligner
    from omnicoder.training.concept_align import ConceptAligner, info_nce, main, triplet
    from omnicoder.training.pre_align import TextEmbedder

    class Flat(torch.nn.Module):
        dim = 16

        def __init__(self):
            super().__init__()
            self.lin = torch.nn.Linear(3, 16)

        def forward(self, x):
            return self.lin(x.mean((2, 3)))

    a = torch.nn.functional.normalize(torch.randn(4, 8), dim=-1)
    assert float(triplet(a, a, -a)) == 0.0 and float(triplet(a, -a, a)) > 2.0
    assert float(info_nce(a * 10, a * 10)) < float(info_nce(a, a.roll(1, 0)))
    torch.manual_seed(0)
    cfg = ModelConfig(name="ca", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64)
    lm = build_model(cfg, "cpu", dtype=torch.float32, seed=0).eval()
    tr = ConceptAligner(lm, ConceptLatentHead(64, 16), TextEmbedder(300, 16), Flat(),
                        PreAligner({"text": 16, "image": 16}, 16), lr=3e-3)
    imgs = torch.rand(6, 3)[:, :, None, None].expand(-1, -1, 4, 4)
    ids = torch.arange(1, 7)[:, None] * torch.tensor([[1, 7, 13]])
    first = tr.step(imgs, ids)
    for _ in range(150):
        last = tr.step(imgs, ids)
    assert last["loss"] < 0.5 * first["loss"]
    assert tr.retrieval_accuracy(imgs, ids) >= 0.8
    assert main(["--steps", "1", "--batch", "4", "--neg_text", "--device", "cpu", "--out",
                 str(tmp_path / "c.pt")]) == 0


def test_unified_mixed_trainer(tmp_path):
    """Mixed rows (image + question, audio + transcript, image + audio + caption, plain text): each
    batch has one modality set, the text-only labels line up with the next token, the loss falls."""
    import json

    from omnicoder.config import AttentionConfig, ModelConfig
    from omnicoder.models.lm import build_model
    from omnicoder.training.tokenizer import get_tokenizer
    from omnicoder.training.vl_tasks import UnifiedMMTrainer, main, unified_example
    torch.manual_seed(0)
    cfg = ModelConfig(name="um", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=128,
                      attn=AttentionConfig(kind="gqa", n_kv_heads=2))
    lm = build_model(cfg, device="cpu", seed=0)
    tok = get_tokenizer(cfg.vocab_size)
    fc = FusionComposer(64, vision=VisionBackbone("vit_tiny", image_size=32, patch=16, depth=1),
                        audio=MelFrontend(out_dim=32))
    torch.save(torch.randn(3, 32, 32), tmp_path / "i.pt")
    torch.save(torch.randn(1600), tmp_path / "a.pt")
    raw = [{"image": str(tmp_path / "i.pt"), "question": "what?", "answer": "a dog"},
           {"audio": str(tmp_path / "a.pt"), "transcript": "hello"},
           {"image": str(tmp_path / "i.pt"), "audio": str(tmp_path / "a.pt"), "caption": "a barking dog"},
           {"text": "just text"}]
    rows = [unified_example(r, 32) for r in raw]
    assert rows[0]["prompt"] == "Question: what? Answer:" and rows[1]["prompt"] == "Transcript:"
    assert sorted(rows[2]["media"]) == ["audio", "image"] and rows[3]["media"] == {}
    with pytest.raises(ValueError):
        unified_example({"image": str(tmp_path / "i.pt")}, 32)
    tr = UnifiedMMTrainer(lm, fc, tok, lr=3e-3)
    b = tr.build({}, [""], ["just text"])                 # text only: position j - 1 predicts token j
    ids = tok.encode("just text") + [tok.eos_id]
    assert b.labels[0, :len(ids) - 1].tolist() == ids[1:] and (b.labels[0, len(ids) - 1:] == -100).all()
    log = tr.fit_mixed(rows, steps=40, batch=2)
    assert {e["modalities"] for e in log} == {"image", "audio", "audio+image", "text"}
    for m in ("image", "text"):
        ls = [e["loss"] for e in log if e["modalities"] == m]
        assert ls[-1] < 0.5 * ls[0], (m, ls)
    (tmp_path / "u.jsonl").write_text("\n".join(json.dumps(r) for r in raw) + "\n")
    assert main(["--task", "unified", "--jsonl", str(tmp_path / "u.jsonl"), "--image_size", "32", "--steps", "2",
                 "--batch", "2", "--device", "cpu", "--out", str(tmp_path / "u.pt")]) == 0


def test_latent_refiner_trained_beside_the_head(tmp_path):
    """--use_refiner: the refiner learns to map the head's estimate to the target, sample() applies it,
    and the checkpoint's refiner runs through the latent-refine tool."""
    import numpy as np

    from omnicoder.config import ModelConfig
    from omnicoder.models.lm import build_model
    from omnicoder.multimodal.video import LatentRefiner
    from omnicoder.tools.utilities import main as tools_main
    from omnicoder.training.flow_recon import FlowReconTrainer, LatentQueryHead, PatchPoolEncoder, main
    torch.manual_seed(0)
    cfg = ModelConfig(name="lr", vocab_size=300, d_model=64, n_layers=2, n_heads=4, ffn_dim=128, max_seq_len=64)
    lm = build_model(cfg, "cpu", dtype=torch.float32, seed=0).eval()
    enc = PatchPoolEncoder(grid=2, channels=8)
    imgs = torch.stack([torch.zeros(3, 16, 16), torch.ones(3, 16, 16)])
    ids = torch.tensor([[5, 6, 7], [8, 9, 10]])
    z0 = enc(imgs)
    ref = LatentRefiner(8)
    tr = FlowReconTrainer(lm, LatentQueryHead(64, 4, 8, width=64), enc, lr=3e-3, refiner=ref)
    losses = [tr.step(imgs, ids) for _ in range(200)]
    assert sum(losses[-10:]) < 0.3 * sum(losses[:10])
    with torch.no_grad():
        raw = tr.head(tr._state(ids))
        assert torch.allclose(tr.sample(ids), ref(raw))
        assert (ref(raw) - z0).norm() / z0.norm() < 0.2
    out = tmp_path / "h.pt"
    assert main(["--steps", "2", "--use_refiner", "--device", "cpu", "--channels", "8", "--out", str(out)]) == 0
    assert "refiner" in torch.load(out, weights_only=False)
    np.save(tmp_path / "z.npy", np.random.default_rng(0).standard_normal((2, 4, 8)).astype(np.float32))
    assert tools_main(["latent-refine", "--latents", str(tmp_path / "z.npy"), "--out_latents",
                       str(tmp_path / "r.npy"), "--ckpt", str(out)]) == 0
