"""CTDG event-stream dataset and batch containers (reference backends/ctdg/runtime/data.py:23-239).

``iter_batches`` walks the split in global windows of ``batch_size * world_size``
events when the stream is partitioned over ranks. With ``assignment ==
"owner"`` (the reference's rule, data.py:172-180) a rank keeps the events whose
source it owns, so per-rank batch sizes follow the skew of the stream (possibly
none: empty batches still take part in every step). With ``"balanced"`` rank r
takes events r, r + W, r + 2W, ... of the window: exactly ``batch_size`` events
per rank. That needs ranks to read and write memory rows of nodes they do not
own, which the NVLink path (remote fetch + push to owners) provides.
``sampler_graph(split)`` returns the events visible to the split: train events
for train, [0, val_end) for val, [0, test_end) for test.
"""
from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Iterator

import torch

from starry_unigraph.data.raw_temporal import load_raw_temporal_events
from starry_unigraph.runtime._split import normalize_split_ratio, split_bounds


@dataclass
class CTDGDataBatch:
    index: int
    split: str
    event_ids: torch.Tensor
    src: torch.Tensor
    dst: torch.Tensor
    ts: torch.Tensor
    edge_feat: torch.Tensor
    src_node_feat: torch.Tensor | None = None
    dst_node_feat: torch.Tensor | None = None

    @property
    def size(self) -> int:
        return int(self.src.numel())

    @property
    def is_empty(self) -> bool:
        return self.size == 0


class TGTemporalDataset:
    def __init__(self, root: str | Path, name: str, split_ratio: dict[str, float] | None = None,
                 config: dict | None = None, raw=None):
        self.root = Path(root).expanduser().resolve() / name
        cfg = dict(config or {})
        cfg.setdefault("data", {})
        cfg["data"] = dict(cfg["data"])
        cfg["data"]["split_ratio"] = split_ratio or cfg["data"].get("split_ratio")
        if raw is None:
            raw = load_raw_temporal_events(root=Path(root).expanduser().resolve(), dataset_name=name, config=cfg)
        self.event_ids = torch.arange(raw.num_edges, dtype=torch.long)
        self.src = raw.src.long()
        self.dst = raw.dst.long()
        self.ts = raw.ts.float()
        self.weight = raw.weight.float() if raw.weight is not None and raw.weight.numel() == raw.src.numel() \
            else torch.ones(raw.src.numel())
        self.num_nodes = int(raw.num_nodes)
        self.num_edges = int(raw.num_edges)
        self.edge_feat = raw.edge_feat if raw.edge_feat.dtype == torch.bfloat16 else raw.edge_feat.float()
        self.edge_feat_dim = int(self.edge_feat.size(-1)) if self.edge_feat.dim() == 2 else 0
        self.node_temporal_features = raw.node_temporal_features
        self.node_feat_dim = 0 if raw.node_temporal_features is None else raw.node_temporal_features.dim
        self.split_ratio = normalize_split_ratio(cfg["data"].get("split_ratio"))
        self._split_cache: dict[str, torch.Tensor] = {}
        self._sampler_cache: dict[str, dict[str, torch.Tensor]] = {}
        self.node_parts: torch.Tensor | None = None
        self.edge_parts: torch.Tensor | None = None
        self.partition_rank = 0
        self.partition_world_size = 1
        self.assignment = "owner"
        self._dst_pool: torch.Tensor | None = None

    def configure_partition(self, *, node_parts, edge_parts, rank: int, world_size: int,
                            assignment: str = "owner") -> None:
        if assignment not in ("owner", "balanced"):
            raise ValueError(f"unknown event assignment {assignment!r} (owner | balanced)")
        self.node_parts = node_parts
        self.edge_parts = edge_parts
        self.partition_rank = rank
        self.partition_world_size = world_size
        self.assignment = assignment

    def split_event_ids(self, split: str) -> torch.Tensor:
        if split not in self._split_cache:
            start, end = split_bounds(self.num_edges, "test" if split == "predict" else split, self.split_ratio)
            self._split_cache[split] = torch.arange(start, end, dtype=torch.long)
        return self._split_cache[split]

    def dst_pool(self) -> torch.Tensor:
        """Unique destinations of the whole stream (negative sampling pool)."""
        if self._dst_pool is None:
            self._dst_pool = torch.unique(self.dst)
        return self._dst_pool

    def lookup_node_features(self, node_ids: torch.Tensor, ts: torch.Tensor) -> torch.Tensor | None:
        table = self.node_temporal_features
        if self.node_feat_dim <= 0 or table is None or table.size == 0:
            return None
        out = torch.zeros(node_ids.numel(), self.node_feat_dim)
        order = torch.argsort(table.node_ids * 0 + table.ts, stable=True)
        ids, tts, vals = table.node_ids[order], table.ts[order], table.values[order]
        for i in range(node_ids.numel()):
            m = (ids == node_ids[i]) & (tts <= ts[i])
            if bool(m.any()):
                out[i] = vals[torch.nonzero(m)[-1, 0]]
        return out

    def global_windows(self, split: str, batch_size: int) -> int:
        indices = self.split_event_ids(split)
        gbs = batch_size * (self.partition_world_size if self.edge_parts is not None else 1)
        return (int(indices.numel()) + gbs - 1) // gbs

    def iter_batches(self, split: str, batch_size: int, start_window: int = 0) -> Iterator[CTDGDataBatch]:
        indices = self.split_event_ids(split)
        distributed = self.partition_world_size > 1 and self.edge_parts is not None
        gbs = batch_size * self.partition_world_size if distributed else batch_size
        for bi, start in enumerate(range(start_window * gbs, int(indices.numel()), gbs), start=start_window):
            ev = indices[start:start + gbs]
            if distributed:
                if self.assignment == "balanced":
                    ev = ev[self.partition_rank::self.partition_world_size]
                else:
                    ev = ev[self.edge_parts[ev] == self.partition_rank]
            s, d, t = self.src[ev], self.dst[ev], self.ts[ev]
            yield CTDGDataBatch(index=bi, split=split, event_ids=ev, src=s, dst=d, ts=t, edge_feat=self.edge_feat[ev],
                                src_node_feat=self.lookup_node_features(s, t) if self.node_feat_dim else None,
                                dst_node_feat=self.lookup_node_features(d, t) if self.node_feat_dim else None)

    def sampler_graph(self, split: str) -> dict[str, torch.Tensor]:
        if split == "predict":
            split = "test"
        if split not in self._sampler_cache:
            _, train_end = split_bounds(self.num_edges, "train", self.split_ratio)
            _, val_end = split_bounds(self.num_edges, "val", self.split_ratio)
            _, test_end = split_bounds(self.num_edges, "test", self.split_ratio)
            end = {"train": train_end, "val": val_end, "test": test_end}.get(split)
            if end is None:
                raise KeyError(f"Unsupported CTDG split: {split}")
            idx = torch.arange(0, end, dtype=torch.long)
            self._sampler_cache[split] = {"row": self.src[idx], "col": self.dst[idx], "eid": idx,
                                          "ts": self.ts[idx].long(), "weight": self.weight[:end]}  # a view: no copy
        return self._sampler_cache[split]

    def describe(self) -> dict[str, int]:
        return {"num_nodes": self.num_nodes, "num_edges": self.num_edges, "edge_feat_dim": self.edge_feat_dim,
                "node_feat_dim": self.node_feat_dim}
