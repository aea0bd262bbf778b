"""Options and result records of the PredictiveLlm facade, and the token odometer.

Reference: PredictiveCoding.LLM/TrainingOptions.cs:27-89, GenerationOptions.cs:6-48,
TrainingReport / GenerationResult / BitsPerByteResult / OnlineLearnReport records,
TokenizerManifest, TokenOdometer.cs:25-95 (unbounded lifetime counters by activity).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

from .generation import SamplingOptions


@dataclass
class TrainingOptions:
    seq_len: int = 32
    stride: int = 16
    epochs: int = 6
    batch_windows: int = 8
    peak_lr: float = 0.01
    min_lr: float = 0.001
    clip_norm: float = 1.0
    held_out_every: int = 5
    max_windows: Optional[int] = None
    on_epoch_end: Optional[Callable[[int, float], None]] = None
    workers: int = 1
    auto_gemm_route: bool = False
    checkpoint_every_steps: int = 0
    checkpoint_dir: Optional[str] = None
    keep_best_by_perplexity: bool = True
    checkpoint_precision: str = "float32"
    resume_optimizer: object = None
    device: Optional[str] = None     # run the autograd step on this device (default: the model's)


@dataclass
class GenerationOptions:
    settle_plan_steps: int = 0
    settle_plan_lr: float = 0.01
    stop_at_eos: bool = True
    learn_from_prompt: bool = False
    sampling: Optional[SamplingOptions] = None
    stop_sequences: Optional[Sequence[str]] = None
    use_memory: bool = False
    memory_top_k: int = 3


@dataclass(frozen=True)
class TrainingReport:
    perplexity_before: float
    perplexity_after: float
    first_loss: float
    last_loss: float
    steps: int
    train_windows: int
    eval_windows: int
    best_perplexity: float = float("nan")
    best_checkpoint_path: Optional[str] = None


@dataclass(frozen=True)
class GenerationResult:
    text: str
    forwards: int
    drafted: int
    accepted: int


@dataclass(frozen=True)
class OnlineLearnReport:
    loss_before: float
    loss_after: float
    steps: int


@dataclass(frozen=True)
class TokenizerManifest:
    kind: str
    vocab_size: int
    hash: str = ""

    def to_json(self) -> bytes:
        return json.dumps({"Kind": self.kind, "VocabSize": self.vocab_size, "Hash": self.hash}).encode()

    @staticmethod
    def from_json(b: bytes) -> "TokenizerManifest":
        d = json.loads(b)
        return TokenizerManifest(d["Kind"], d["VocabSize"], d.get("Hash", ""))


class TokenOdometer:
    """Lifetime logical token counters (Python ints never roll over)."""

    FIELDS = ("trained", "evaluated", "absorbed", "prompted", "generated")

    def __init__(self):
        self.reset()

    def reset(self) -> None:
        for f in self.FIELDS:
            setattr(self, f, 0)

    @property
    def total(self) -> int:
        return sum(getattr(self, f) for f in self.FIELDS)

    def add_served(self, prompted: int, generated: int) -> None:
        if prompted < 0 or generated < 0:
            raise ValueError("An odometer only goes forward.")
        self.prompted += prompted
        self.generated += generated

    def to_json(self) -> bytes:
        return json.dumps({f.capitalize(): getattr(self, f) for f in self.FIELDS}).encode()

    def load_json(self, b: bytes) -> None:
        d = json.loads(b)
        for f in self.FIELDS:
            setattr(self, f, int(d.get(f.capitalize(), 0)))

    def __str__(self) -> str:
        return (f"tokens: {self.total:,} total | trained {self.trained:,} · evaluated {self.evaluated:,} · "
                f"absorbed {self.absorbed:,} · prompted {self.prompted:,} · generated {self.generated:,}")
