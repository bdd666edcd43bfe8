"""Per-partition cache of halo rows keyed by (snapshot, partition)
(reference runtime/cache/partition_cache.py, a stub)."""
from __future__ import annotations

from typing import Any

from torch import Tensor


class PartitionCache:
    def __init__(self, capacity: int = 64):
        self.capacity = int(capacity)
        self.store: dict[tuple[int, int], Tensor] = {}
        self.order: list[tuple[int, int]] = []

    def get(self, snapshot: int, part: int) -> Tensor | None:
        return self.store.get((snapshot, part))

    def put(self, snapshot: int, part: int, rows: Tensor) -> None:
        key = (snapshot, part)
        if key not in self.store:
            self.order.append(key)
        self.store[key] = rows
        while len(self.order) > self.capacity:
            self.store.pop(self.order.pop(0), None)

    def describe(self) -> dict[str, Any]:
        return {"entries": len(self.store), "capacity": self.capacity}
