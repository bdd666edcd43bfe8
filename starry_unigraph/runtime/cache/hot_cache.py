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
        """(hit mask, rows): a sorted search of the resident ids, at any capacity; hits
        count toward their slot's frequency, misses read as zero rows."""
        ids = node_ids.to(self.ids.device).long().view(-1)
        hit = torch.zeros(ids.numel(), dtype=torch.bool, device=ids.device)
        out = torch.zeros(ids.numel(), self.rows.size(1), dtype=self.rows.dtype, device=self.rows.device)
        occupied = torch.nonzero(self.ids >= 0).view(-1)
        if occupied.numel() and ids.numel():
            key, order = torch.sort(self.ids[occupied])
            pos = torch.searchsorted(key, ids).clamp(max=key.numel() - 1)
            hit = key[pos] == ids
            slot = occupied[order[pos[hit]]]
            out[hit] = self.rows[slot]
            self.freq.index_add_(0, slot, torch.ones_like(slot))
        self.hits += int(hit.sum())
        self.misses += int((~hit).sum())
        return hit, out

    def insert(self, node_ids: Tensor, rows: Tensor) -> None:
        """Insert or refresh rows in one pass: ids already cached are updated in
        place (frequency + 1), new ids take the least-frequently used slots (at
        most `capacity` of them, the last occurrence of a repeated id wins)."""
        ids = node_ids.to(self.ids.device).long().view(-1)
        rows = rows.to(self.rows)
        if ids.numel() == 0:
            return
        # last occurrence of every id in the batch
        uniq, inverse = torch.unique(ids, return_inverse=True)
        last = torch.full((uniq.numel(),), -1, dtype=torch.long, device=ids.device)
        last.scatter_reduce_(0, inverse, torch.arange(ids.numel(), device=ids.device), reduce="amax")
        ids, rows = uniq, rows[last]
        # ids already resident: sorted search over the occupied slot ids
        occupied = torch.nonzero(self.ids >= 0).view(-1)
        present = torch.zeros(ids.numel(), dtype=torch.bool, device=ids.device)
        if occupied.numel():
            key, order = torch.sort(self.ids[occupied])
            pos = torch.searchsorted(key, ids).clamp(max=key.numel() - 1)
            present = key[pos] == ids
            slots = occupied[order[pos[present]]]
            self.rows[slots] = rows[present]
            self.freq[slots] += 1
        fresh_ids, fresh_rows = ids[~present], rows[~present]
        take = min(fresh_ids.numel(), self.capacity)
        if take:
            # least-frequently used slots first (free slots have frequency 0)
            victims = torch.topk(self.freq, take, largest=False).indices
            self.ids[victims] = fresh_ids[:take]
            self.rows[victims] = fresh_rows[:take]
            self.freq[victims] = 1

    def clear(self) -> None:
        self.ids.fill_(-1)
        self.freq.zero_()

    def describe(self) -> dict[str, Any]:
        return {"capacity": self.capacity, "occupied": int((self.ids >= 0).sum()), "hits": self.hits,
                "misses": self.misses}
