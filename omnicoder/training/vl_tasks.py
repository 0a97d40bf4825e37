"""Vision / audio / video - language task trainers over the fusion composer.

Reference: src/omnicoder/training/ vl_fused_pretrain.py, vqa_fused_train.py,
coco_captions_train.py, video_vqa_train.py, ocr_train.py, asr_train.py (one trainer
per task, each composing modality features with the prompt and training the language
model to produce the answer).  Here one `VLTaskTrainer` holds the recipe and the tasks
differ by their prompt template and input modality:

  vl_pretrain   image  ->  description (loss on every text token)
  vqa           image + "Question: ... Answer:"  ->  answer
  caption       image + "Caption:"               ->  caption
  ocr           image + "Text in the image:"     ->  text
  video_qa      video + question                 ->  answer
  asr           audio + "Transcript:"            ->  transcript

A step: the prompt + target token ids are embedded by the LM, the composer puts the
modality's projected features (with begin / end markers) in front, the LM runs on the
composed embeddings, and the cross entropy counts only the target tokens (modality,
marker and prompt positions are ignored; `loss_on_prompt` counts the prompt too).
JSONL rows: {"image" | "video" | "audio": path to a tensor file (.pt / .npy) or an
image file, "question", "answer" | "caption" | "text" | "transcript"}.
"""
from __future__ import annotations

import json
from dataclasses import dataclass

import torch

TASKS = {
    "vl_pretrain": ("image", "", "caption"),
    "vqa": ("image", "Question: {question} Answer:", "answer"),
    "caption": ("image", "Caption:", "caption"),
    "ocr": ("image", "Text in the image:", "text"),
    "video_qa": ("video", "Question: {question} Answer:", "answer"),
    "asr": ("audio", "Transcript:", "transcript"),
}


def load_media(path: str, image_size: int = 224) -> torch.Tensor:
    """A tensor file (.pt / .npy) as saved, or an image file as [3, S, S] in [-1, 1]."""
    if path.endswith(".pt"):
        return torch.load(path, weights_only=True)
    if path.endswith(".npy"):
        import numpy as np
        return torch.from_numpy(np.load(path))
    from PIL import Image
    import numpy as np
    img = Image.open(path).convert("RGB").resize((image_size, image_size))
    return torch.from_numpy(np.asarray(img)).permute(2, 0, 1).float() / 127.5 - 1.0


def read_task_jsonl(path: str, task: str, limit: int = 0) -> list[dict]:
    modality, template, key = TASKS[task]
    rows = []
    with open(path) as f:
        for line in f:
            if not line.strip():
                continue
            r = json.loads(line)
            rows.append({"media": load_media(r[modality]), "prompt": template.format(**r), "target": r[key]})
            if limit and len(rows) >= limit:
                break
    return rows


@dataclass
class VLBatch:
    embeds: torch.Tensor      # [B, L, D] composed inputs
    labels: torch.Tensor      # [B, L] next-token targets, -100 where not trained


class VLTaskTrainer:
    def __init__(self, lm, composer, tokenizer, task: str, lr: float = 1e-4, train_lm: bool = True,
                 loss_on_prompt: bool = False):
        if task not in TASKS:
            raise ValueError(f"unknown task {task!r}; one of {sorted(TASKS)}")
        self.lm, self.composer, self.tok, self.task = lm, composer, tokenizer, task
        self.modality = TASKS[task][0]
        self.loss_on_prompt = loss_on_prompt
        params = list(composer.parameters()) + (list(lm.parameters()) if train_lm else [])
        if not train_lm:
            for p in lm.parameters():
                p.requires_grad_(False)
        self.opt = torch.optim.AdamW([p for p in params if p.requires_grad], lr=lr)

    def build(self, media, prompts: list[str], targets: list[str]) -> VLBatch:
        """Compose one batch (prompt / target pairs padded to the longest with ignored positions).
        `media`: a tensor of the task's modality, or {modality: tensor} for any subset of image,
        video and audio (empty for text-only rows)."""
        dev = self.lm.embed.device
        seqs, masks = [], []
        for p, t in zip(prompts, targets):
            pi = self.tok.encode(p) if p else []
            ti = self.tok.encode(" " + t if p else t) + [self.tok.eos_id if hasattr(self.tok, "eos_id") else 0]
            seqs.append(pi + ti)
            masks.append([self.loss_on_prompt] * len(pi) + [True] * len(ti))
        T = max(len(s) for s in seqs)
        ids = torch.zeros(len(seqs), T, dtype=torch.long)
        train = torch.zeros(len(seqs), T, dtype=torch.bool)
        for b, (s, m) in enumerate(zip(seqs, masks)):
            ids[b, :len(s)] = torch.tensor(s)
            train[b, :len(s)] = torch.tensor(m)
        ids, train = ids.to(dev), train.to(dev)
        text_emb = self.lm.embed[ids]
        kw = media if isinstance(media, dict) else {self.modality: media}
        emb, seg = self.composer.fuse_all(text_emb, **{k: v.to(dev) for k, v in kw.items() if v is not None})
        n_pre = emb.shape[1] - T                     # modality tokens + markers in front of the text
        labels = torch.full(emb.shape[:2], -100, dtype=torch.long, device=dev)
        # position n_pre - 1 + j predicts text token j (without media, token 0 has no predictor)
        tgt = torch.where(train, ids, torch.full_like(ids, -100))
        first = 1 if n_pre == 0 else 0
        labels[:, n_pre - 1 + first:n_pre - 1 + T] = tgt[:, first:]
        return VLBatch(emb, labels)

    def step(self, media: torch.Tensor, prompts: list[str], targets: list[str]) -> float:
        b = self.build(media, prompts, targets)
        out = self.lm(None, labels=b.labels, embeds=b.embeds)
        out["ce"].backward()
        self.opt.step()
        self.opt.zero_grad(set_to_none=True)
        return float(out["ce"].detach())

    def fit(self, rows: list[dict], steps: int, batch: int = 4) -> list[float]:
        losses = []
        for i in range(steps):
            chunk = [rows[(i * batch + j) % len(rows)] for j in range(batch)]
            media = torch.stack([r["media"] for r in chunk])
            losses.append(self.step(media, [r["prompt"] for r in chunk], [r["target"] for r in chunk]))
        return losses

    @torch.no_grad()
    def answer(self, media: torch.Tensor, prompt: str, max_new_tokens: int = 16) -> str:
        """Greedy answer for one input (full forward per token; evaluation helper)."""
        dev = self.lm.embed.device
        ids = self.tok.encode(prompt) if prompt else []
        out = []
        for _ in range(max_new_tokens):
            cur = torch.tensor([ids + out], dtype=torch.long, device=dev)
            emb, _ = self.composer.fuse_all(self.lm.embed[cur], **{self.modality: media[None].to(dev)})
            logits = self.lm(None, embeds=emb, all_logits=True)["logits"][0, -1]
            out.append(int(logits.argmax()))
        return self.tok.decode(out)


_PROMPTS = (("question", "Question: {question} Answer:", "answer"), ("caption", "Caption:", "caption"),
            ("transcript", "Transcript:", "transcript"), ("text", "", "text"))


def unified_example(row: dict, image_size: int = 224) -> dict:
    """A mixed-corpus row (the reference's unified multimodal trainer, src/omnicoder/training/
    unified_multimodal_train.py:44-120: any subset of image / video / audio paths with a question +
    answer, a caption, a transcript or plain text) -> {"media": {modality: tensor}, "prompt", "target"}.
    The target is the first of answer (with its question), caption, transcript, text present."""
    media = {m: load_media(row[m], image_size) for m in ("image", "video", "audio") if isinstance(row.get(m), str)}
    for key, template, tkey in _PROMPTS:
        if row.get(tkey) and (key != "question" or row.get("question")):
            return {"media": media, "prompt": template.format(**row), "target": str(row[tkey])}
    raise ValueError(f"row has no target (answer, caption, transcript or text): {sorted(row)}")


class UnifiedMMTrainer(VLTaskTrainer):
    """One model over mixed rows: each batch holds rows with the same set of modalities (so their
    features stack), and the cross entropy counts the target text only."""

    def __init__(self, lm, composer, tokenizer, lr: float = 1e-4, train_lm: bool = True, loss_on_prompt: bool = False):
        super().__init__(lm, composer, tokenizer, "vl_pretrain", lr, train_lm, loss_on_prompt)

    def fit_mixed(self, rows: list[dict], steps: int, batch: int = 4) -> list[dict]:
        groups: dict = {}
        for r in rows:
            groups.setdefault(tuple(sorted(r["media"])), []).append(r)
        keys = sorted(groups)
        log = []
        for i in range(steps):
            key = keys[i % len(keys)]
            g = groups[key]
            chunk = [g[(i // len(keys) * batch + j) % len(g)] for j in range(min(batch, len(g)))]
            media = {m: torch.stack([r["media"][m] for r in chunk]) for m in key}
            loss = self.step(media, [r["prompt"] for r in chunk], [r["target"] for r in chunk])
            log.append({"modalities": "+".join(key) or "text", "loss": loss})
        return log


def synthetic_rows(task: str, n: int, image_size: int = 64, seed: int = 0) -> list[dict]:
    """Rows of random media with templated questions / targets (wiring and throughput runs)."""
    g = torch.Generator().manual_seed(seed)
    modality, template, _ = TASKS[task]
    rows = []
    for i in range(n):
        if modality == "image":
            media = torch.rand(3, image_size, image_size, generator=g) * 2 - 1
        elif modality == "video":
            media = torch.rand(4, 3, image_size, image_size, generator=g) * 2 - 1
        else:
            media = torch.randn(16000, generator=g) * 0.1
        rows.append({"media": media, "prompt": template.format(question=f"what is item {i}?"), "target": f"item {i}"})
    return rows


def main(argv=None):
    import argparse

    from ..config import get_preset
    from ..models.lm import build_model
    from ..multimodal.backbones import VisionBackbone
    from ..multimodal.composer import FusionComposer
    from ..multimodal.encoders import MelFrontend
    from ..multimodal.video import VideoEncoder
    from .tokenizer import get_tokenizer
    ap = argparse.ArgumentParser(description="vision / audio / video - language task training")
    ap.add_argument("--task", default="vqa", choices=sorted(TASKS) + ["unified"],
                    help="unified: mixed rows with any subset of image / video / audio and a text target")
    ap.add_argument("--jsonl", default="", help="task rows (default: synthetic rows)")
    ap.add_argument("--preset", default="tiny_moe")
    ap.add_argument("--vision", default="vit_tiny")
    ap.add_argument("--image_size", type=int, default=64)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--batch", type=int, default=4)
    ap.add_argument("--lr", type=float, default=1e-4)
    ap.add_argument("--out", default="weights/vl.pt")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    a = ap.parse_args(argv)
    dev = torch.device(a.device)
    lm = build_model(get_preset(a.preset), device=dev, dtype=torch.float32, seed=0)
    D = lm.cfg.d_model
    comp = FusionComposer(D, vision=VisionBackbone(a.vision, image_size=a.image_size, depth=2),
                          video=VideoEncoder(image_size=a.image_size, dim=192, depth=1, heads=3),
                          audio=MelFrontend(out_dim=D)).to(dev)
    tok = get_tokenizer(lm.cfg.vocab_size)
    if a.task == "unified":
        tr = UnifiedMMTrainer(lm, comp, tok, lr=a.lr)
        if a.jsonl:
            with open(a.jsonl) as f:
                rows = [unified_example(json.loads(ln), a.image_size) for ln in f if ln.strip()]
        else:
            rows = [dict(r, media={TASKS[t][0]: r["media"]}) for t in ("vqa", "asr", "video_qa")
                    for r in synthetic_rows(t, 2 * a.batch, a.image_size)]
            rows += [{"media": {}, "prompt": "", "target": f"plain text row {i}"} for i in range(a.batch)]
        losses = [e["loss"] for e in tr.fit_mixed(rows, a.steps, a.batch)]
    else:
        tr = VLTaskTrainer(lm, comp, tok, a.task, lr=a.lr)
        rows = read_task_jsonl(a.jsonl, a.task) if a.jsonl else synthetic_rows(a.task, 4 * a.batch, a.image_size)
        losses = tr.fit(rows, a.steps, a.batch)
    torch.save({"model": lm.export_state_dict(), "composer": comp.state_dict(), "config": lm.cfg.to_dict()}, a.out)
    print(json.dumps({"task": a.task, "steps": a.steps, "first_loss": losses[0], "last_loss": losses[-1],
                      "out": a.out}))
    return 0


if __name__ == "__main__":
    main()
