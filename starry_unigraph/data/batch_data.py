"""Unified batch container (reference data/batch_data.py:15-42)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

from torch import Tensor


@dataclass
class BatchData:
    """Graph structure (``mfg``: a message-flow graph, here a plain CSR/dense
    sampling block), node ids, and task-specific fields."""

    mfg: Any
    node_ids: Tensor
    pos_src: Tensor | None = None
    pos_dst: Tensor | None = None
    neg_src: Tensor | None = None
    neg_dst: Tensor | None = None
    target_nodes: Tensor | None = None
    labels: Tensor | None = None
    timestamps: Tensor | None = None
    chunk_id: tuple | None = None
    local_node_mask: Tensor | None = None
    remote_manifest: dict[str, Any] | None = None
    nbr_feat: Tensor | None = None  # [roots, k, F] feature rows of the sampled neighbours (ChunkAtomic.complete)
    source: Any = None  # the unit (ChunkAtomic) the batch was materialised from
