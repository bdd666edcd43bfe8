"""Same-time-slice communication plan between clusters (reference runtime/comm/spatial_plan.py)."""
from __future__ import annotations

from dataclasses import dataclass, field

from torch import Tensor


@dataclass
class SpatialPlan:
    send_ids: dict[int, Tensor] = field(default_factory=dict)   # peer rank -> ids to send
    recv_ids: dict[int, Tensor] = field(default_factory=dict)   # peer rank -> ids to receive

    def volume(self) -> int:
        return int(sum(t.numel() for t in self.send_ids.values()))
