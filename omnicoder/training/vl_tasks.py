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
