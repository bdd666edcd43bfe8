"""MemShare-style historical cache (reference backends/ctdg/runtime/cache.py:18-180).

Caches the last value pushed for every shared (non-owned) node; a new update is
only pushed when the cosine distance to the cached value exceeds 1 - alpha, so a
larger alpha pushes more rows. ``AdaParameter`` moves alpha with the ratio of a
step's sync time to its compute time; the host runtime drives it after every
training step when ``ctdg.ada_param_enabled`` is set.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.nn.functional as F


@dataclass
class AdaParameter:
    alpha: float = 0.5
    min_alpha: float = 0.1
    max_alpha: float = 0.95
    _step: int = field(default=0, init=False, repr=False)

    def update_from_latency(self, sync_ms: float, compute_ms: float) -> None:
        """Push fewer rows when sync outweighs compute, more when compute does.

        alpha moves by 0.01 * (1 - sync / compute) per call, within [min_alpha,
        max_alpha]. The reference (cache.py:26-37) adds 0.01 * (ratio - 1), which
        raises alpha, and so the number of pushed rows, exactly when its own comment
        says sync dominates and filtering should tighten; this keeps the documented
        intent (the reference never calls the method)."""
        if compute_ms <= 0:
            return
        ratio = sync_ms / (compute_ms + 1e-9)
        self.alpha = float(max(self.min_alpha, min(self.max_alpha, self.alpha + 0.01 * (1.0 - ratio))))
        self._step += 1


class CTDGHistoricalCache:
    def __init__(self, num_shared: int, hidden_dim: int, device: str, num_nodes: int | None = None,
                 shared_node_ids: torch.Tensor | None = None, ada_param: AdaParameter | None = None) -> None:
        self.num_shared = num_shared
        self.hidden_dim = hidden_dim
        self.device = device
        self.ada_param = ada_param or AdaParameter()
        self._cached_memory = torch.zeros(num_shared, hidden_dim, dtype=torch.float32, device=device)
        self._cached_memory_ts = torch.full((num_shared,), -1.0, dtype=torch.float32, device=device)
        self._slot_by_global: torch.Tensor | None = None
        if num_nodes is not None and shared_node_ids is not None:
            self.bind_shared_nodes(num_nodes, shared_node_ids)

    def bind_shared_nodes(self, num_nodes: int, shared_node_ids: torch.Tensor) -> None:
        slot = torch.full((num_nodes,), -1, dtype=torch.long, device=self.device)
        ids = shared_node_ids.long().to(self.device)
        if ids.numel():
            slot[ids] = torch.arange(ids.numel(), dtype=torch.long, device=self.device)
        self._slot_by_global = slot

    def slot_indices(self, node_ids: torch.Tensor) -> torch.Tensor:
        if self._slot_by_global is None:
            return torch.full(node_ids.shape, -1, dtype=torch.long, device=self.device)
        ids = node_ids.long().to(self.device)
        ok = (ids >= 0) & (ids < self._slot_by_global.numel())
        out = torch.full(ids.shape, -1, dtype=torch.long, device=self.device)
        out[ok] = self._slot_by_global[ids[ok]]
        return out

    def historical_check(self, node_ids: torch.Tensor, current_memory: torch.Tensor) -> torch.Tensor:
        """True where the node drifted beyond the threshold (or was never cached)."""
        if node_ids.numel() == 0:
            return torch.zeros(0, dtype=torch.bool, device=self.device)
        slots = self.slot_indices(node_ids)
        valid = slots >= 0
        cached = self._cached_memory[slots.clamp(min=0)]
        never = self._cached_memory_ts[slots.clamp(min=0)] < 0
        dist = 1.0 - F.cosine_similarity(current_memory.to(self.device).float(), cached, dim=1)
        return (dist > (1.0 - self.ada_param.alpha)) | ~valid | never

    def update_cache(self, slots: torch.Tensor, new_memory: torch.Tensor, new_ts: torch.Tensor) -> None:
        slots = slots.long().to(self.device)
        keep = slots >= 0
        if bool(keep.any()):
            self._cached_memory[slots[keep]] = new_memory.float().to(self.device)[keep]
            self._cached_memory_ts[slots[keep]] = new_ts.float().to(self.device)[keep]

    def synchronize_shared_update(self, node_ids: torch.Tensor, values: torch.Tensor, ts: torch.Tensor) -> None:
        slots = self.slot_indices(node_ids)
        keep = slots >= 0
        if not bool(keep.any()):
            return
        s, v, t = slots[keep], values.float().to(self.device)[keep], ts.float().to(self.device)[keep]
        newer = t > self._cached_memory_ts[s]
        self._cached_memory[s[newer]] = v[newer]
        self._cached_memory_ts[s[newer]] = t[newer]
