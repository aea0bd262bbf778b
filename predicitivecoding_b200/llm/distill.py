"""Sequence-level distillation from a teacher function, and the on-policy (SEED-style) round.

Reference: PredictiveCoding.LLM/Training/LmDistiller.cs:29-166.  ``build_dataset`` asks the
teacher for the completion of every prompt (optionally cached on disk as JSONL); ``step``
trains on prompt + completion with the loss masked to the completion; ``on_policy_round``
lets the student draft, asks the teacher for a corrected completion, and trains on it.
"""
from __future__ import annotations

import hashlib
import json
import os
from typing import Callable, List, Optional, Sequence, Tuple

import torch

from ..optim.adam import Adam
from .generation import greedy
from .trainer import step as adam_step


def build_dataset(prompts: Sequence[str], teacher: Callable[[str], str],
                  cache_dir: Optional[str] = None) -> List[Tuple[str, str]]:
    out = []
    cache = {}
    path = None
    if cache_dir:
        os.makedirs(cache_dir, exist_ok=True)
        path = os.path.join(cache_dir, "teacher.jsonl")
        if os.path.exists(path):
            for line in open(path, encoding="utf-8"):
                d = json.loads(line)
                cache[d["key"]] = d["completion"]
    for p in prompts:
        k = hashlib.sha256(p.encode("utf-8")).hexdigest()[:16]
        if k not in cache:
            cache[k] = teacher(p)
            if path:
                with open(path, "a", encoding="utf-8") as f:
                    f.write(json.dumps({"key": k, "prompt": p, "completion": cache[k]}) + "\n")
        out.append((p, cache[k]))
    return out


def _example(tok, prompt: str, completion: str, max_seq: int):
    pids = tok.encode(prompt, add_bos=True)
    cids = tok.encode(completion, add_eos=True)
    full = (pids + cids)[: max_seq + 1]
    tokens = full[:-1]
    targets = full[1:]
    for i in range(min(len(pids) - 1, len(targets))):
        targets[i] = -1
    return tokens, targets


def step(model, tok, data, optimizer: Adam, lr: float, clip_norm: float = 1.0) -> float:
    batch = [_example(tok, p, c, model.cfg.max_seq) for p, c in data]
    return adam_step(list(model.parameters()), batch,
                     lambda t, y, tr: model.loss(t.view(1, -1), y.view(1, -1), -1, tr), optimizer, lr, clip_norm)


def on_policy_round(model, tok, prompts: Sequence[str], teacher_correct: Callable[[str, str], str],
                    optimizer: Adam, lr: float, draft_tokens: int = 16, clip_norm: float = 1.0) -> float:
    data = []
    for p in prompts:
        ids = tok.encode(p, add_bos=True)
        out = greedy(model, ids, draft_tokens, tok.eos)
        draft = tok.decode(out[len(ids):])
        data.append((p, teacher_correct(p, draft)))
    return step(model, tok, data, optimizer, lr, clip_norm)
