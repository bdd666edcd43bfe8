"""Node / edge feature storage (reference data/feature_store.py:15-68, a protocol
only there).

``FeatureStore`` is the reference's read interface: features of this rank's
owned nodes by global id, edge features by event id, the owned-node count,
feature widths and ``pin_memory`` for asynchronous host-to-device copies.
``TensorFeatureStore`` implements it over named dense tables: node tables are
indexed through the sorted owned-id list (a global id that this rank does not
own raises ``IndexError``), edge tables directly by event id. On CUDA the tables
live in HBM and reads are gathers; on the host they can be pinned so that
``to(device, non_blocking=True)`` overlaps compute. Remote reads are not its
job: the runtimes fetch remote rows over NVLink or NCCL themselves.
"""
from __future__ import annotations

from typing import Protocol

import torch
from torch import Tensor


class FeatureStore(Protocol):
    def get_node_feat(self, node_ids: Tensor, feat_name: str = "x") -> Tensor: ...

    def get_edge_feat(self, edge_ids: Tensor, feat_name: str = "edge_attr") -> Tensor: ...

    def num_nodes(self) -> int: ...

    def feat_dim(self, feat_name: str = "x") -> int: ...

    def pin_memory(self) -> "FeatureStore": ...


class TensorFeatureStore:
    """Named [rows, F] tables. ``node_ids`` lists the global id of each node-table row
    (default: row i is node i, every node owned)."""

    def __init__(self, node_feat: Tensor | dict[str, Tensor] | None = None,
                 edge_feat: Tensor | dict[str, Tensor] | None = None, node_ids: Tensor | None = None):
        if isinstance(node_feat, Tensor):
            node_feat = {"x": node_feat}
        if isinstance(edge_feat, Tensor):
            edge_feat = {"edge_attr": edge_feat}
        self.node_tables: dict[str, Tensor] = dict(node_feat or {})
        self.edge_tables: dict[str, Tensor] = dict(edge_feat or {})
        rows = {int(t.size(0)) for t in self.node_tables.values()}
        if len(rows) > 1:
            raise ValueError(f"node tables disagree on their row count: {sorted(rows)}")
        self._rows = rows.pop() if rows else (0 if node_ids is None else int(node_ids.numel()))
        self._sorted_ids: Tensor | None = None
        self._row_of_sorted: Tensor | None = None
        if node_ids is not None:
            ids = node_ids.long().view(-1)
            if ids.numel() != self._rows:
                raise ValueError(f"{ids.numel()} node ids for {self._rows} table rows")
            self._sorted_ids, self._row_of_sorted = torch.sort(ids)

    # ------------------------------------------------------------------ reads
    def _rows_of(self, node_ids: Tensor, device: torch.device) -> Tensor:
        ids = node_ids.to(device).long().view(-1)
        if self._sorted_ids is None:
            bad = (ids < 0) | (ids >= self._rows)
            if bool(bad.any()):
                raise IndexError(f"node id {int(ids[bad][0])} is not owned by this store")
            return ids
        key = self._sorted_ids.to(device)
        pos = torch.searchsorted(key, ids).clamp(max=max(key.numel() - 1, 0))
        found = key[pos] == ids if key.numel() else torch.zeros_like(ids, dtype=torch.bool)
        if not bool(found.all()):
            raise IndexError(f"node id {int(ids[~found][0])} is not owned by this store")
        return self._row_of_sorted.to(device)[pos]

    def get_node_feat(self, node_ids: Tensor, feat_name: str = "x") -> Tensor:
        table = self.node_tables[feat_name]  # KeyError for an unknown name
        return table[self._rows_of(node_ids, table.device)]

    def get_edge_feat(self, edge_ids: Tensor, feat_name: str = "edge_attr") -> Tensor:
        table = self.edge_tables[feat_name]
        return table[edge_ids.to(table.device).long()]

    # ------------------------------------------------------------------ writes
    def put_node_feat(self, node_ids: Tensor, values: Tensor, feat_name: str = "x") -> None:
        table = self.node_tables[feat_name]
        table[self._rows_of(node_ids, table.device)] = values.to(table)

    # ------------------------------------------------------------------ shape / placement
    def num_nodes(self) -> int:
        return self._rows

    def feat_dim(self, feat_name: str = "x") -> int:
        table = self.node_tables.get(feat_name, self.edge_tables.get(feat_name))
        if table is None:
            raise KeyError(feat_name)
        return int(table.size(1)) if table.dim() > 1 else 1

    def pin_memory(self) -> "TensorFeatureStore":
        """Host tables to page-locked memory (a no-op for device tables and where no
        CUDA runtime is available); returns self."""
        if torch.cuda.is_available():
            for tables in (self.node_tables, self.edge_tables):
                for k, t in tables.items():
                    if t.device.type == "cpu" and not t.is_pinned():
                        tables[k] = t.pin_memory()
        return self

    def to(self, device: str | torch.device, non_blocking: bool = False) -> "TensorFeatureStore":
        """Copy of the store with every table on `device` (asynchronous from pinned memory)."""
        out = TensorFeatureStore({k: t.to(device, non_blocking=non_blocking) for k, t in self.node_tables.items()},
                                 {k: t.to(device, non_blocking=non_blocking) for k, t in self.edge_tables.items()})
        out._rows = self._rows
        if self._sorted_ids is not None:
            out._sorted_ids = self._sorted_ids.to(device, non_blocking=non_blocking)
            out._row_of_sorted = self._row_of_sorted.to(device, non_blocking=non_blocking)
        return out

    # ------------------------------------------------------------------ compatibility
    def get(self, node_ids: Tensor) -> Tensor:
        return self.get_node_feat(node_ids)

    def put(self, node_ids: Tensor, values: Tensor) -> None:
        self.put_node_feat(node_ids, values)

    @property
    def dim(self) -> int:
        return self.feat_dim("x")
