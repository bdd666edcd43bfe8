"""Cross-time state dependency plan (reference module runtime/comm/state_plan.py,
a placeholder there): for a training window, which carried-state rows each
slot reads and how many rows the window writes back."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch
from torch import Tensor


@dataclass
class StatePlan:
    read_versions: dict[int, Tensor] = field(default_factory=dict)   # window slot -> state rows read
    write_nodes: Tensor | None = None                                # rows of the newest snapshot

    @classmethod
    def from_window(cls, blob: Any) -> "StatePlan":
        """Rows each slot of a frozen window (``STGraphBlob``) reads from the
        carried state: its graph's destination rows."""
        plan = cls()
        for step in blob.steps:
            plan.read_versions[int(step.slot)] = torch.arange(int(step.graph.num_dst_nodes))
        if blob.steps:
            plan.write_nodes = torch.arange(int(blob.steps[-1].graph.num_dst_nodes))
        return plan

    def describe(self) -> dict:
        return {"reads": {k: int(v.numel()) for k, v in self.read_versions.items()},
                "writes": 0 if self.write_nodes is None else int(self.write_nodes.numel())}
