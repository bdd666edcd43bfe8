"""Same-time-slice communication plan between partitions (reference module
runtime/comm/spatial_plan.py, a placeholder there): which rows each peer sends
and receives for one snapshot, derived from the snapshot's halo route."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch
from torch import Tensor


@dataclass
class SpatialPlan:
    send_ids: dict[int, Tensor] = field(default_factory=dict)   # peer rank -> local rows sent to it
    recv_ids: dict[int, Tensor] = field(default_factory=dict)   # peer rank -> halo slots filled from it

    @classmethod
    def from_route(cls, route: Any) -> "SpatialPlan":
        """Per-peer rows of a halo route: send rows are the route's send_index
        split by ``send_sizes``; received rows are the halo slots in ``recv_sizes``
        order (slot 0 = the first row after the local rows)."""
        plan = cls()
        if route is None or route.send_index is None:
            return plan
        send = torch.split(route.send_index.long().cpu(), [int(s) for s in route.send_sizes])
        start = 0
        for peer, (rows, n_recv) in enumerate(zip(send, route.recv_sizes)):
            if rows.numel():
                plan.send_ids[peer] = rows
            if int(n_recv):
                plan.recv_ids[peer] = torch.arange(start, start + int(n_recv))
            start += int(n_recv)
        return plan

    def volume(self) -> int:
        """Rows this rank sends."""
        return int(sum(t.numel() for t in self.send_ids.values()))

    def received(self) -> int:
        return int(sum(t.numel() for t in self.recv_ids.values()))
