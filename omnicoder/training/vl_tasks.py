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

    def build(self, media: torch.Tensor, prompts: list[str], targets: list[str]) -> VLBatch:
        """Compose one batch (prompt / target pairs padded to the longest with ignored positions)."""
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
        emb, seg = self.composer.fuse_all(text_emb, **{self.modality: media.to(dev)})
        n_pre = emb.shape[1] - T                     # modality tokens + markers in front of the text
        labels = torch.full(emb.shape[:2], -100, dtype=torch.long, device=dev)
        # position n_pre - 1 + j predicts text token j
        tgt = torch.where(train, ids, torch.full_like(ids, -100))
        labels[:, n_pre - 1:n_pre - 1 + T] = tgt
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
    ap.add_argument("--task", default="vqa", choices=sorted(TASKS))
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
    tr = VLTaskTrainer(lm, comp, get_tokenizer(lm.cfg.vocab_size), a.task, lr=a.lr)
    rows = read_task_jsonl(a.jsonl, a.task) if a.jsonl else synthetic_rows(a.task, 4 * a.batch, a.image_size)
    losses = tr.fit(rows, a.steps, a.batch)
    torch.save({"model": lm.export_state_dict(), "composer": comp.state_dict(), "config": lm.cfg.to_dict()}, a.out)
    print(json.dumps({"task": a.task, "steps": a.steps, "first_loss": losses[0], "last_loss": losses[-1],
                      "out": a.out}))
    return 0


if __name__ == "__main__":
    main()
