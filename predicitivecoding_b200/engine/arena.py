"""Flat parameter arena: one fp32 master / grad / Adam-moment buffer and one bf16
working copy, with named views, laid out for sharding across data-parallel ranks.

The reference keeps a separate device allocation per parameter tensor and runs
one AdamW launch per tensor (PredictiveCoding.Device/Training/DeviceDecoderTrainer.cs:545-557).
One flat buffer lets a single kernel update everything, lets gradient
reduce-scatter operate on contiguous shards, and keeps every tensor 64-element
aligned (128-byte aligned in bf16), which TMA descriptors require.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple

import torch

ALIGN = 64  # elements


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


@dataclass
class ParamSpec:
    name: str
    shape: Tuple[int, ...]
    decay: bool = True

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= s
        return n


class ParamArena:
    """Offsets of named tensors inside flat buffers.

    Decayed tensors come first, so AdamW can apply weight decay to the prefix
    ``[0, n_decay)``.  The total is padded to ``world * shard`` so every rank
    owns one contiguous, aligned shard.
    """

    def __init__(self, specs: Sequence[ParamSpec], world: int = 1):
        specs = [s for s in specs if s.decay] + [s for s in specs if not s.decay]
        self.specs: List[ParamSpec] = list(specs)
        self.offsets: Dict[str, int] = {}
        off = 0
        self.n_decay = 0
        for s in self.specs:
            self.offsets[s.name] = off
            off += _round_up(s.numel, ALIGN)
            if s.decay:
                self.n_decay = off
        self.used = off
        self.world = world
        self.shard = _round_up((off + world - 1) // world, ALIGN)
        self.total = self.shard * world
        self.by_name = {s.name: s for s in self.specs}

    def view(self, flat: torch.Tensor, name: str) -> torch.Tensor:
        s = self.by_name[name]
        o = self.offsets[name]
        return flat[o:o + s.numel].view(*s.shape)

    def views(self, flat: torch.Tensor) -> Dict[str, torch.Tensor]:
        return {s.name: self.view(flat, s.name) for s in self.specs}

    @property
    def numel(self) -> int:
        return sum(s.numel for s in self.specs)
