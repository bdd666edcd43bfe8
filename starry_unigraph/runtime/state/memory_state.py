"""Three-tier node-memory state for CTDG (reference runtime/state/memory_state.py:26,
a stub there): owned rows live in the memory bank, a hot cache keeps frequently
read remote rows, a decay cache keeps recently fetched rows for a few versions."""
from __future__ import annotations

from typing import Any

import torch
from torch import Tensor

from starry_unigraph.runtime.cache.decay_cache import DecayCache
from starry_unigraph.runtime.cache.hot_cache import HotCache


class CTDGStateManager:
    def __init__(self, memory_bank: Any, hot_capacity: int = 4096, decay_versions: int = 2):
        self.bank = memory_bank
        self.hot = HotCache(hot_capacity, memory_bank.hidden_dim, memory_bank.memory.device)
        self.decay = DecayCache(decay_versions)
        self.version = 0

    def prepare(self, node_ids: Tensor, timestamps: Tensor | None = None) -> dict[str, Any]:
        ids = node_ids.to(self.bank.memory.device).long()
        mem = self.bank.gather(ids)
        owned = self.bank.is_owned(ids)
        if not bool(owned.all()):
            rem = ~owned
            hit, rows = self.hot.lookup(ids[rem])
            if bool(hit.any()):
                sub = mem[rem]
                sub[hit] = rows[hit]
                mem[rem] = sub
        return {"memory": mem, "mailbox": self.bank.read_mailbox(ids), "version": self.version}

    def patch(self, node_ids: Tensor, rows: Tensor) -> None:
        self.hot.insert(node_ids, rows)
        self.decay.put(self.version, node_ids, rows)

    def update(self, model_output: dict[str, Tensor], chunk: Any) -> None:
        if "memory_ids" in model_output and "memory_rows" in model_output:
            ts = model_output.get("memory_ts")
            ids = model_output["memory_ids"]
            self.bank._apply_memory_update(ids, model_output["memory_rows"],
                                           ts if ts is not None else torch.zeros(ids.numel()))

    def step(self) -> None:
        self.version += 1
        self.decay.expire(self.version)

    def reset(self) -> None:
        self.hot.clear()
        self.decay.clear()
        self.version = 0

    def describe(self) -> dict[str, Any]:
        return {"manager": "ctdg_memory", "version": self.version, "hot": self.hot.describe(),
                "decay": self.decay.describe()}
