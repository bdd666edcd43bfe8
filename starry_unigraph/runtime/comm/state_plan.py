"""Cross-time state dependency plan (reference runtime/comm/state_plan.py)."""
from __future__ import annotations

from dataclasses import dataclass, field

from torch import Tensor


@dataclass
class StatePlan:
    read_versions: dict[int, Tensor] = field(default_factory=dict)   # version -> nodes read
    write_nodes: Tensor | None = None

    def describe(self) -> dict:
        return {"reads": {k: int(v.numel()) for k, v in self.read_versions.items()},
                "writes": 0 if self.write_nodes is None else int(self.write_nodes.numel())}
