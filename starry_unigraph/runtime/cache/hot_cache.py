"""Device-resident cache of frequently read remote node rows with
least-frequently-used eviction (reference runtime/cache/hot_cache.py, a stub)."""
from __future__ import annotations

from typing import Any

import torch
from torch import Tensor


class HotCache:
    def __init__(self, capacity: int, dim: int, device: Any = "cpu"):
        self.capacity = int(capacity)
        self.rows = torch.zeros(self.capacity, dim, device=device)
        self.ids = torch.full((self.capacity,), -1, dtype=torch.long, device=device)
        self.freq = torch.zeros(self.capacity, dtype=torch.long, device=device)
        self.hits = 0
        self.misses = 0

    def lookup(self, node_ids: Tensor) -> tuple[Tensor, Tensor]:
        ids = node_ids.to(self.ids.device).long()
        match = ids.unsqueeze(1) == self.ids.unsqueeze(0) if self.capacity <= 65536 else None
        if match is None:
            return torch.zeros_like(ids, dtype=torch.bool), torch.zeros(ids.numel(), self.rows.size(1))
        hit = match.any(1)
        slot = match.float().argmax(1)
        self.freq.index_add_(0, slot[hit], torch.ones_like(slot[hit]))
        self.hits += int(hit.sum())
        self.misses += int((~hit).sum())
        return hit, self.rows[slot]

    def insert(self, node_ids: Tensor, rows: Tensor) -> None:
        ids = node_ids.to(self.ids.device).long()
        for i in range(ids.numel()):
            present = torch.nonzero(self.ids == ids[i])
            slot = int(present[0]) if present.numel() else int(torch.argmin(self.freq))
            self.ids[slot] = ids[i]
            self.rows[slot] = rows[i].to(self.rows)
            self.freq[slot] = self.freq[slot] + 1 if present.numel() else 1

    def clear(self) -> None:
        self.ids.fill_(-1)
        self.freq.zero_()

    def describe(self) -> dict[str, Any]:
        return {"capacity": self.capacity, "occupied": int((self.ids >= 0).sum()), "hits": self.hits,
                "misses": self.misses}
