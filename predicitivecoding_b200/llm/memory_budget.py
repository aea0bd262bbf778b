"""Training-memory estimate for a decoder configuration, measured from one real forward/backward.

Reference: PredictiveCoding.LLM/Training/MemoryBudget.cs:24-110 (parameters, gradients = parameters,
Adam m+v = 2x parameters, activations = every non-parameter tensor reachable from the loss with its
gradient; the fp16 projection halves weights-copy, gradients and activations and keeps fp32
masters and Adam states).  Activations here are the tensors autograd saves for the backward
(counted once each, with an equal-sized gradient), measured by a saved-tensor hook.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models.config import DecoderLmConfig
from ..models.decoder_lm import DecoderLM


def _gb(b: int) -> str:
    return f"{b / 1024 ** 3:.2f} GB"


@dataclass(frozen=True)
class MemoryBudgetReport:
    config: DecoderLmConfig
    seq_len: int
    parameter_bytes: int
    gradient_bytes: int
    adam_state_bytes: int
    activation_bytes: int

    @property
    def total_bytes(self) -> int:
        return self.parameter_bytes + self.gradient_bytes + self.adam_state_bytes + self.activation_bytes

    @property
    def project_fp16_bytes(self) -> int:
        return (self.parameter_bytes // 2 + self.parameter_bytes + self.gradient_bytes // 2 + self.adam_state_bytes
                + self.activation_bytes // 2)

    def describe(self) -> str:
        return (f"seq {self.seq_len}, params {_gb(self.parameter_bytes)} + grads {_gb(self.gradient_bytes)} "
                f"+ adam {_gb(self.adam_state_bytes)} + activations {_gb(self.activation_bytes)} "
                f"= {_gb(self.total_bytes)} fp32  (fp16 projection {_gb(self.project_fp16_bytes)})")


def measure(cfg: DecoderLmConfig, seq_len: int, seed: int = 42) -> MemoryBudgetReport:
    if not 2 <= seq_len <= cfg.max_seq:
        raise ValueError(f"seq_len ({seq_len}) must be in [2, max_seq {cfg.max_seq}].")
    model = DecoderLM(cfg, seed=seed)
    params = list(model.parameters())
    pbytes = sum(p.numel() * 4 for p in params)
    pids = {p.data_ptr() for p in params}
    g = torch.Generator().manual_seed(seed + 1)
    tokens = torch.randint(0, cfg.vocab, (1, seq_len), generator=g)
    targets = torch.roll(tokens, -1, 1)
    seen = set()
    act = [0]

    def pack(t):
        key = (t.data_ptr(), t.numel(), t.dtype)
        if t.data_ptr() not in pids and key not in seen:
            seen.add(key)
            act[0] += t.numel() * t.element_size() * 2      # value + its gradient
        return t

    with torch.autograd.graph.saved_tensors_hooks(pack, lambda t: t):
        loss = model.loss(tokens, targets, -1, True)
    loss.backward()
    return MemoryBudgetReport(cfg, seq_len, pbytes, pbytes, 2 * pbytes, act[0])
