"""Seeded synthetic data of the benchmark shapes (no network datasets in this environment)."""
from __future__ import annotations

import numpy as np
import torch


def zipf_tokens(n: int, vocab: int, s: float = 1.1, seed: int = 0) -> torch.Tensor:
    """i.i.d. token ids drawn from a Zipf(s) law over ``vocab`` symbols (rank 1 = id 0)."""
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    p = ranks ** (-s)
    p /= p.sum()
    ids = rng.choice(vocab, size=n, p=p)
    return torch.from_numpy(ids.astype(np.int64))


def zipf_windows(batch: int, seq: int, vocab: int, s: float = 1.1, seed: int = 0):
    """[batch, seq] inputs and next-token targets cut from one Zipf stream."""
    t = zipf_tokens(batch * (seq + 1), vocab, s, seed).view(batch, seq + 1)
    return t[:, :-1].contiguous(), t[:, 1:].contiguous()
