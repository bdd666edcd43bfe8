"""Task-specific sampling configuration (reference data/sample_config.py:15-41)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

from torch import Tensor


@dataclass
class SampleConfig:
    """Controls what a batch materialises. Edge prediction uses ``pos_src`` /
    ``pos_dst``; node tasks use ``target_nodes`` / ``target_labels``."""

    pos_src: Tensor | None = None
    pos_dst: Tensor | None = None
    neg_strategy: str = "none"  # "cache_aware" | "random" | "none"
    neg_ratio: int = 1
    target_nodes: Tensor | None = None
    target_labels: Tensor | None = None
    num_neighbors: list[int] = field(default_factory=lambda: [20, 10])
    num_layers: int = 2
    sample_type: str = "temporal"  # "temporal" | "random"
    extra: dict[str, Any] = field(default_factory=dict)
