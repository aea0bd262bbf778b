"""Continual learning: absorb text online with surprise-scaled learning rate, replay and a drift guard.

Reference: PredictiveCoding.LLM/Training/ContinualLearner.cs:29-231.  Each ``absorb`` builds the
text's windows, scales the base lr by surprise = loss_before / EMA(loss) clamped to
[min_lr_scale, max_lr_scale], trains ``steps`` Adam steps on fresh + a rotating replay slice,
pushes the fresh windows into a ring replay buffer, and every ``guardrail_every`` absorbs compares
a yardstick perplexity against its baseline, calling ``on_drift`` past ``drift_threshold``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch

from ..optim.adam import Adam
from .data import StreamingTextDataset
from .eval import evaluate as perplexity
from .trainer import step as adam_step


@dataclass(frozen=True)
class ContinualOptions:
    seq_len: int = 32
    stride: int = 16
    base_lr: float = 0.002
    steps: int = 1
    clip_norm: float = 1.0
    replay_capacity: int = 128
    replay_per_step: int = 4
    min_lr_scale: float = 0.25
    max_lr_scale: float = 4.0
    surprise_ema_decay: float = 0.9
    guardrail_every: int = 0
    drift_threshold: float = 0.25


@dataclass(frozen=True)
class ContinualStep:
    surprise_before: float
    surprise_after: float
    effective_lr: float
    replay_windows: int


@dataclass(frozen=True)
class ContinualDrift:
    baseline_perplexity: float
    current_perplexity: float
    relative_drift: float
    absorb_count: int


class ContinualLearner:
    def __init__(self, llm, options: Optional[ContinualOptions] = None, yardstick_text: Optional[str] = None):
        self.llm = llm
        self.opts = options or ContinualOptions()
        self.seq_len = min(self.opts.seq_len, llm.config.max_seq)
        self.optimizer = Adam()
        self.replay: List[Tuple[list, list]] = []
        self.replay_cursor = 0
        self.surprise_avg = -1.0
        self.absorb_count = 0
        self.on_drift: Optional[Callable[[ContinualDrift], None]] = None
        self.yardstick = self._windows(yardstick_text) if yardstick_text else None
        self.baseline_perplexity = (perplexity(llm.model, self.yardstick).perplexity
                                    if self.yardstick else float("nan"))

    @property
    def replay_size(self) -> int:
        return len(self.replay)

    def measure_yardstick(self) -> float:
        return perplexity(self.llm.model, self.yardstick).perplexity if self.yardstick else float("nan")

    def _windows(self, text: str):
        return list(StreamingTextDataset(text.split("\n"), self.llm.tokenizer, self.seq_len, self.opts.stride).windows())

    def _whole(self, text: str):
        tok = self.llm.tokenizer
        ids = tok.encode(text, add_bos=True)
        if len(ids) < 2:
            ids = [tok.bos] + ids + [tok.eos]
        n = min(len(ids) - 1, self.seq_len)
        return ids[:n], ids[1:n + 1]

    def _loss_fn(self, t, y, training):
        return self.llm.model.loss(t.view(1, -1), y.view(1, -1), -1, training)

    def _mean_loss(self, ws) -> float:
        m = self.llm.model
        dev = next(m.parameters()).device
        with torch.no_grad():
            return sum(float(m.loss(torch.tensor([t], device=dev), torch.tensor([y], device=dev), -1, False))
                       for t, y in ws) / len(ws)

    def _take_replay(self, n: int):
        if self.opts.replay_capacity == 0 or n <= 0 or not self.replay:
            return []
        out = []
        for _ in range(min(n, len(self.replay))):
            self.replay_cursor = (self.replay_cursor + 1) % len(self.replay)
            out.append(self.replay[self.replay_cursor])
        return out

    def _push_replay(self, ws) -> None:
        cap = self.opts.replay_capacity
        if cap == 0:
            return
        for w in ws:
            if len(self.replay) < cap:
                self.replay.append(w)
            else:
                self.replay[self.replay_cursor % cap] = w
                self.replay_cursor = (self.replay_cursor + 1) % cap

    def absorb(self, text: str) -> ContinualStep:
        o = self.opts
        fresh = self._windows(text) or [self._whole(text)]
        before = self._mean_loss(fresh)
        scale = 1.0
        if o.surprise_ema_decay > 0:
            if self.surprise_avg < 0:
                self.surprise_avg = before
            scale = min(max(before / max(self.surprise_avg, 1e-6), o.min_lr_scale), o.max_lr_scale)
        lr = o.base_lr * scale
        replay = self._take_replay(o.replay_per_step)
        batch = fresh + replay
        params = list(self.llm.model.parameters())
        for _ in range(o.steps):
            adam_step(params, batch, self._loss_fn, self.optimizer, lr, o.clip_norm)
        after = self._mean_loss(fresh)
        self._push_replay(fresh)
        if o.surprise_ema_decay > 0:
            self.surprise_avg = o.surprise_ema_decay * self.surprise_avg + (1 - o.surprise_ema_decay) * before
        self.absorb_count += 1
        self._guardrail()
        return ContinualStep(before, after, lr, len(replay))

    def _guardrail(self) -> None:
        o = self.opts
        if o.guardrail_every <= 0 or not self.yardstick or self.absorb_count % o.guardrail_every:
            return
        now = self.measure_yardstick()
        drift = (now - self.baseline_perplexity) / self.baseline_perplexity
        if drift > o.drift_threshold and self.on_drift is not None:
            self.on_drift(ContinualDrift(self.baseline_perplexity, now, drift, self.absorb_count))
