"""Long-running GPU pretraining loop: hashed train/held-out split, warmup + cosine lr, periodic
held-out evaluation, bits-per-byte probe and samples, rolling and best checkpoints (model in the
reference checkpoint layout + DAM1 Adam state), JSONL progress log and resume.

Reference: PredictiveCoding.Device/Training/DevicePretrainer.cs:1-279 (DevicePretrainOptions,
DevicePretrainProgress, DevicePretrainReport, ``Pretrain``).  Same schedule and bookkeeping; the
step runs the fused sm_100a trainer when the model fits its contract (dense RMSNorm/RoPE decoder on
a GPU) and the autograd step of the facade otherwise.
"""
from __future__ import annotations

import json
import math
import os
import time
from dataclasses import dataclass
from typing import Callable, List, Optional

import torch

from ..llm.data import StreamingTextDataset
from ..llm.eval import held_out_hashed, training_split_hashed


@dataclass(frozen=True)
class DevicePretrainOptions:
    epochs: int = 1
    seq_len: int = 512
    stride: int = 512
    micro_batch_windows: int = 4
    peak_lr: float = 3e-4
    min_lr: float = 3e-5
    warmup_steps: int = 100
    total_steps: int = 0
    max_steps: int = 0
    weight_decay: float = 0.01
    held_out_every: int = 10
    eval_windows: int = 64
    eval_every_steps: int = 200
    quality_every_steps: int = 0
    sample_prompt: str = "The"
    sample_tokens: int = 48
    checkpoint_dir: Optional[str] = None
    checkpoint_every_steps: int = 1000
    keep_best_checkpoint: bool = True
    log_path: Optional[str] = None
    on_progress: Optional[Callable] = None


@dataclass(frozen=True)
class DevicePretrainProgress:
    epoch: int
    step: int
    lr: float
    train_loss: float
    eval_loss: Optional[float]
    bits_per_byte: Optional[float]
    sample: Optional[str]
    best_eval_loss: float
    tokens: int
    tokens_per_second: float
    wall_seconds: float
    eta_seconds: Optional[float]


@dataclass(frozen=True)
class DevicePretrainReport:
    steps: int
    tokens: int
    final_train_loss: float
    final_eval_loss: float
    best_eval_loss: float
    final_bits_per_byte: Optional[float]
    elapsed_seconds: float
    checkpoint_dir: Optional[str]
    best_checkpoint_dir: Optional[str]


def lr_at(step: int, horizon: int, o: DevicePretrainOptions) -> float:
    if o.warmup_steps > 0 and step <= o.warmup_steps:
        return o.peak_lr * step / o.warmup_steps
    if horizon <= 0:
        return o.peak_lr
    if step >= horizon:
        return o.min_lr
    t = (step - o.warmup_steps) / max(1, horizon - o.warmup_steps)
    return o.min_lr + (o.peak_lr - o.min_lr) * 0.5 * (1 + math.cos(math.pi * t))


class _Stepper:
    """Fused GPU trainer when possible, the facade's autograd step otherwise."""

    def __init__(self, llm, o: DevicePretrainOptions):
        from ..engine.fused_trainer import FusedDecoderTrainer, supports
        self.llm = llm
        self.fused = None
        dev = next(llm.model.parameters()).device
        if dev.type == "cuda" and supports(llm.config, o.seq_len):
            self.fused = FusedDecoderTrainer(llm.config, o.micro_batch_windows, o.seq_len, device=dev,
                                             lr=o.peak_lr, weight_decay=o.weight_decay, model=llm.model,
                                             use_graph=True)
        else:
            from ..optim.adam import Adam
            self.opt = Adam(weight_decay=o.weight_decay)

    def step(self, batch, lr: float) -> float:
        if self.fused is not None:
            tok = torch.tensor([w[0] for w in batch])
            tgt = torch.tensor([w[1] for w in batch])
            return self.fused.step(tok, tgt, lr)
        from ..llm.trainer import step as adam_step
        m = self.llm.model
        return adam_step(list(m.parameters()), batch,
                         lambda t, y, tr: m.loss(t.view(1, -1), y.view(1, -1), -1, tr), self.opt, lr, 1.0)

    def eval_loss(self, windows) -> float:
        if not windows:
            return float("nan")
        if self.fused is not None:
            B = self.fused.B
            tot, n = 0.0, 0
            for i in range(0, len(windows) - B + 1, B):
                chunk = windows[i:i + B]
                tot += self.fused.evaluate_loss(torch.tensor([w[0] for w in chunk]),
                                                torch.tensor([w[1] for w in chunk])) * len(chunk)
                n += len(chunk)
            if n:
                return tot / n
        m = self.llm.model
        dev = next(m.parameters()).device
        with torch.no_grad():
            return sum(float(m.loss(torch.tensor([t], device=dev), torch.tensor([y], device=dev), -1, False))
                       for t, y in windows) / len(windows)

    def export(self) -> None:
        if self.fused is not None:
            self.fused.export_model(self.llm.model)

    def save_state(self, path: str) -> None:
        if self.fused is not None:
            self.fused.save_state(path)

    def load_state(self, path: str) -> None:
        if self.fused is not None and os.path.exists(path):
            self.fused.load_state(path)


def _append_log(path: str, p: DevicePretrainProgress) -> None:
    d = os.path.dirname(path)
    if d:
        os.makedirs(d, exist_ok=True)
    rec = {"step": p.step, "epoch": p.epoch, "lr": p.lr, "trainLoss": p.train_loss}
    if p.eval_loss is not None:
        rec["evalLoss"] = p.eval_loss
    if p.bits_per_byte is not None:
        rec["bitsPerByte"] = p.bits_per_byte
    rec.update({"tokens": p.tokens, "tokPerSec": round(p.tokens_per_second, 1), "wallSeconds": round(p.wall_seconds, 1)})
    with open(path, "a") as f:
        f.write(json.dumps(rec) + "\n")


def pretrain(llm, corpus, options: Optional[DevicePretrainOptions] = None, cancel: Optional[Callable[[], bool]] = None
             ) -> DevicePretrainReport:
    o = options or DevicePretrainOptions()
    if o.seq_len > llm.config.max_seq:
        raise ValueError(f"seq_len {o.seq_len} exceeds the model's max_seq {llm.config.max_seq}.")
    cancel = cancel or (lambda: False)
    stepper = _Stepper(llm, o)
    ck = o.checkpoint_dir
    adam_path = os.path.join(ck, "adam-device.bin") if ck else None
    best_dir = os.path.join(ck, "best") if ck and o.keep_best_checkpoint else None
    if adam_path:
        stepper.load_state(adam_path)

    def windows():
        return StreamingTextDataset(corpus.lines(), llm.tokenizer, o.seq_len, o.stride).windows()

    held = list(held_out_hashed(windows(), o.held_out_every))[: o.eval_windows]
    probe = "".join(llm.tokenizer.decode(t) + "\n" for _, t in held[:4])
    horizon = o.total_steps if o.total_steps > 0 else o.max_steps
    t0 = time.perf_counter()
    step = tokens = 0
    train_loss = eval_loss = float("nan")
    best = float("inf")
    last_bits = None
    batch: List = []
    stop = False
    for epoch in range(o.epochs):
        if stop or cancel():
            break
        for w in training_split_hashed(windows(), o.held_out_every):
            if stop or cancel():
                break
            if len(w[0]) != o.seq_len:
                continue
            batch.append(w)
            if len(batch) < o.micro_batch_windows:
                continue
            step += 1
            lr = lr_at(step, horizon, o)
            train_loss = stepper.step(batch, lr)
            tokens += sum(len(b[0]) for b in batch)
            batch = []
            eval_due = bool(held) and o.eval_every_steps > 0 and step % o.eval_every_steps == 0
            quality_due = o.quality_every_steps > 0 and step % o.quality_every_steps == 0
            ckpt_due = ck is not None and o.checkpoint_every_steps > 0 and step % o.checkpoint_every_steps == 0
            if eval_due:
                eval_loss = stepper.eval_loss(held)
            new_best = eval_due and best_dir is not None and eval_loss < best
            bits = sample = None
            if quality_due or ckpt_due or new_best:
                stepper.export()
                if quality_due:
                    bits = llm.evaluate_bits_per_byte(probe).bits_per_byte if probe else None
                    last_bits = bits
                    try:
                        sample = llm.generate(o.sample_prompt, o.sample_tokens).replace("\n", " ").strip()
                    except Exception:
                        sample = "(generation failed)"
                if new_best:
                    best = eval_loss
                    llm.save(best_dir)
                    stepper.save_state(os.path.join(best_dir, "adam-device.bin"))
                if ckpt_due:
                    llm.save(ck)
                    stepper.save_state(adam_path)
            wall = time.perf_counter() - t0
            eta = (horizon - step) * wall / step if horizon > 0 and step < horizon else None
            prog = DevicePretrainProgress(epoch, step, lr, train_loss, eval_loss if eval_due else None, bits, sample,
                                          best if best < float("inf") else float("nan"), tokens,
                                          tokens / max(1e-9, wall), wall, eta)
            if o.log_path:
                _append_log(o.log_path, prog)
            if o.on_progress:
                o.on_progress(prog)
            if o.max_steps > 0 and step >= o.max_steps:
                stop = True
    if batch and not stop and not cancel() and stepper.fused is None:
        step += 1
        train_loss = stepper.step(batch, lr_at(step, horizon, o))
        tokens += sum(len(b[0]) for b in batch)
    if held:
        eval_loss = stepper.eval_loss(held)
    stepper.export()
    if ck:
        llm.save(ck)
        stepper.save_state(adam_path)
    return DevicePretrainReport(step, tokens, train_loss, eval_loss, best if best < float("inf") else eval_loss,
                                last_bits, time.perf_counter() - t0, ck, best_dir)
