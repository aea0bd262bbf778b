"""Episodic memory: a bounded cosine-similarity key/value store of remembered texts.

Reference: PredictiveCoding.LLM/Training/EpisodicMemory.cs:23-156 (capacity-bounded FIFO of
(key, text) pairs, recall = top-k by cosine similarity) used by PredictiveLlm.Remember and
recall-into-generation; PredicitiveCoding/Networks/Memory/MemoryBank.cs for the PC analogue.
"""
from __future__ import annotations

from collections import deque
from typing import List, Sequence, Tuple

import torch


class EpisodicMemory:
    def __init__(self, key_dim: int, capacity: int = 1024):
        if key_dim <= 0 or capacity <= 0:
            raise ValueError("key_dim and capacity must be positive")
        self.key_dim, self.capacity = key_dim, capacity
        self._items: deque = deque(maxlen=capacity)

    def __len__(self) -> int:
        return len(self._items)

    @property
    def count(self) -> int:
        return len(self._items)

    def remember(self, key: Sequence[float], text: str) -> None:
        k = torch.as_tensor(key, dtype=torch.float32).flatten().cpu()
        if k.numel() != self.key_dim:
            raise ValueError(f"key has {k.numel()} dims, memory expects {self.key_dim}")
        self._items.append((k, text))

    def recall(self, query: Sequence[float], top_k: int = 3) -> List[Tuple[str, float]]:
        if not self._items:
            return []
        q = torch.as_tensor(query, dtype=torch.float32).flatten().cpu()
        K = torch.stack([k for k, _ in self._items])
        sims = torch.nn.functional.cosine_similarity(K, q[None], dim=-1)
        top = torch.topk(sims, min(top_k, len(self._items)))
        return [(self._items[i][1], float(s)) for s, i in zip(top.values.tolist(), top.indices.tolist())]

    def live_entries_oldest_first(self) -> List[Tuple[torch.Tensor, str]]:
        return list(self._items)
