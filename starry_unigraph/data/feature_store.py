"""Feature storage protocol and an in-device implementation
(reference data/feature_store.py:15-68)."""
from __future__ import annotations

from typing import Protocol

import torch
from torch import Tensor


class FeatureStore(Protocol):
    def get(self, node_ids: Tensor) -> Tensor: ...

    def put(self, node_ids: Tensor, values: Tensor) -> None: ...

    @property
    def dim(self) -> int: ...


class TensorFeatureStore:
    """Dense [N, F] feature table on one device (HBM-resident on CUDA)."""

    def __init__(self, table: Tensor):
        self.table = table

    def get(self, node_ids: Tensor) -> Tensor:
        return self.table[node_ids.to(self.table.device).long()]

    def put(self, node_ids: Tensor, values: Tensor) -> None:
        self.table[node_ids.to(self.table.device).long()] = values.to(self.table)

    @property
    def dim(self) -> int:
        return int(self.table.size(1))
