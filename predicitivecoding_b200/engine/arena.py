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
from typing import Dict, List, Optional, Sequence, Tuple

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

    Unbucketed (``buckets=None``): decayed tensors come first, so AdamW can apply
    weight decay to the prefix ``[0, n_decay)``, and the total is padded to
    ``world * shard`` so every rank owns one contiguous, aligned shard.

    Bucketed (``buckets`` = lists of tensor names, in the order their gradients
    become final during the backward): each bucket is a contiguous range
    (decayed tensors first, then the rest) padded to a multiple of
    ``world * ALIGN`` and split into ``world`` equal pieces; rank ``r`` owns piece
    ``r`` of every bucket, and its local optimizer state is those pieces back to
    back (``pieces(r)``).  Every bucket's gradient can then be reduce-scattered as
    soon as the backward has produced it, with every rank receiving an equal part.
    """

    def __init__(self, specs: Sequence[ParamSpec], world: int = 1,
                 buckets: Optional[Sequence[Sequence[str]]] = None):
        self.world = world
        self.by_name = {s.name: s for s in specs}
        self.offsets: Dict[str, int] = {}
        self.buckets: List[Tuple[int, int, int]] = []   # (start, end, decay_end) in the flat buffer
        if buckets is None:
            specs = [s for s in specs if s.decay] + [s for s in specs if not s.decay]
            self.specs: List[ParamSpec] = list(specs)
            off = 0
            self.n_decay = 0
            for s in self.specs:
                self.offsets[s.name] = off
                off += _round_up(s.numel, ALIGN)
                if s.decay:
                    self.n_decay = off
            self.used = off
            self.shard = _round_up((off + world - 1) // world, ALIGN)
            self.total = self.shard * world
            return
        names = [n for b in buckets for n in b]
        if sorted(names) != sorted(s.name for s in specs) or len(set(names)) != len(names):
            raise ValueError("buckets must name every tensor exactly once")
        self.specs = []
        off = 0
        for b in buckets:
            start = off
            group = [self.by_name[n] for n in b]
            group = [s for s in group if s.decay] + [s for s in group if not s.decay]
            decay_end = start
            for s in group:
                self.specs.append(s)
                self.offsets[s.name] = off
                off += _round_up(s.numel, ALIGN)
                if s.decay:
                    decay_end = off
            off = start + _round_up(off - start, world * ALIGN)
            self.buckets.append((start, off, decay_end))
        self.used = off
        self.total = off
        self.shard = off // world
        self.n_decay = -1   # not a prefix: use the per-bucket decay ends

    def pieces(self, rank: int) -> List[Tuple[int, int, int, int]]:
        """This rank's pieces of the bucketed layout: (local offset, flat start, length, flat decay end)."""
        if not self.buckets:
            lo = rank * self.shard
            return [(0, lo, self.shard, self.n_decay)]
        out, loff = [], 0
        for start, end, dend in self.buckets:
            c = (end - start) // self.world
            out.append((loff, start + rank * c, c, dend))
            loff += c
        return out

    def gather_local(self, flat: torch.Tensor, rank: int) -> torch.Tensor:
        """Rank ``rank``'s shard of a full flat buffer, in local order."""
        return torch.cat([flat[g:g + n] for _, g, n, _ in self.pieces(rank)])

    def scatter_local(self, local: torch.Tensor, rank: int, flat: torch.Tensor) -> None:
        """Write rank ``rank``'s local shard back into its places in a full flat buffer."""
        for lo, g, n, _ in self.pieces(rank):
            flat[g:g + n].copy_(local[lo:lo + n])

    def view(self, flat: torch.Tensor, name: str) -> torch.Tensor:
        s = self.by_name[name]
        o = self.offsets[name]
        return flat[o:o + s.numel].view(*s.shape)

    def views(self, flat: torch.Tensor) -> Dict[str, torch.Tensor]:
        return {s.name: self.view(flat, s.name) for s in self.specs}

    @property
    def numel(self) -> int:
        return sum(s.numel for s in self.specs)
