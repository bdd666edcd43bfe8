"""Flare runtime loader: splits, chunk order / decay, iteration
(reference backends/dtdg/runtime/session_loader.py:27-341).

Training yields ``STGraphBlob`` windows; evaluation / prediction replay the
snapshots from the start one by one, marking snapshots before the split as
``snapshot_warmup`` (they only advance the carried RNN state).
``chunk_order`` accepts ``rand`` and ``random`` (the reference's default value
``random`` is not recognised there and silently means identity order).
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Any, Iterable

import torch

from starry_unigraph.data.partition import PartitionData
from starry_unigraph.runtime._split import normalize_split_ratio, split_bounds

from .loader import STGraphLoader
from .state import STGraphBlob


@dataclass
class SnapshotRoutePlan:
    route_type: str
    cache_policy: str

    def describe(self) -> dict[str, Any]:
        return asdict(self) | {"type": "SnapshotRoutePlan"}


@dataclass
class DTDGWindowState:
    window_size: int
    last_snapshot: int | None = None
    stored_windows: int = 0

    def store(self, snapshot_index: int) -> None:
        self.last_snapshot = snapshot_index
        self.stored_windows += 1

    def describe(self) -> dict[str, Any]:
        return asdict(self)


@dataclass
class DTDGBatch:
    index: int
    split: str
    window_size: int
    route_plan: SnapshotRoutePlan
    adjacency: list[list[float]]
    dense_features: list[float]
    graph: Any = None
    graph_meta: dict[str, Any] = field(default_factory=dict)
    chain: str = "load_snapshot->route_apply->state_fetch->state_transition->state_writeback"

    def to_payload(self) -> dict[str, Any]:
        return {"index": self.index, "split": self.split, "chain": self.chain,
                "window": {"snapshot_id": self.index, "window_size": self.window_size},
                "route_plan": self.route_plan.describe(), "adjacency": self.adjacency,
                "dense_features": self.dense_features, "graph_meta": self.graph_meta}


def _parse_chunk_order(mode: Any, chunk_count: int, generator: torch.Generator | None = None):
    if chunk_count <= 0 or mode in (None, "none"):
        return None
    if mode in ("rand", "random"):
        return torch.randperm(chunk_count, generator=generator)
    if mode == "reverse":
        return torch.arange(chunk_count - 1, -1, -1)
    return torch.arange(chunk_count)


def _parse_chunk_decay(value: Any, chunk_count: int) -> list[int]:
    if chunk_count <= 0 or value in (None, "none", [], ()):
        return []
    if isinstance(value, int):
        return list(range(1, max(1, min(chunk_count, value)) + 1))
    if isinstance(value, (list, tuple)):
        return sorted({max(1, min(chunk_count, int(v))) for v in value})
    if value == "half":
        return [max(1, chunk_count // 2)]
    if value == "all":
        return list(range(1, chunk_count + 1))
    return []


def _block_to_batch(block, split: str, window_size: int, route_plan: SnapshotRoutePlan) -> DTDGBatch:
    blob_meta = None
    if isinstance(block, STGraphBlob):
        blob_meta = block.describe()
        block = block.current_graph
    n_edges = max(1, block.num_edges())
    local_src = int((block.edge_src < block.num_dst_nodes).sum())
    x = block.dstdata.get("x", block.srcdata.get("x"))
    mean_x = x.float().mean(0) if x is not None and x.numel() else torch.zeros(2)
    dense = [float(mean_x[0]), float(mean_x[1]) if mean_x.numel() > 1 else 0.0]
    return DTDGBatch(index=int(block.graph_meta.get("snapshot_index", getattr(block, "flare_snapshot_id", 0))),
                     split=split, window_size=window_size, route_plan=route_plan,
                     adjacency=[[local_src / n_edges, (block.num_edges() - local_src) / n_edges],
                                [block.num_dst_nodes / max(1, block.num_src_nodes), 1.0]],
                     dense_features=dense, graph=block,
                     graph_meta={"num_src_nodes": block.num_src_nodes, "num_dst_nodes": block.num_dst_nodes,
                                 "num_edges": block.num_edges(),
                                 "flare_is_full_snapshot": bool(getattr(block, "flare_is_full_snapshot", True)),
                                 "window_blob": blob_meta})


@dataclass
class FlareRuntimeLoader:
    partition_id: int
    route_plan: SnapshotRoutePlan
    window_state: DTDGWindowState
    partition_data: PartitionData
    graph_loader: STGraphLoader
    device: str
    rank: int
    world_size: int
    chunk_index: torch.Tensor
    train_chunk_order: Any = None
    train_chunk_decay: list[int] = field(default_factory=list)
    train_num_full_snaps: int = 1
    split_ratio: dict[str, float] | None = None
    cursor: int = 0
    window_from_size: bool = False
    seed: int = 0

    def __post_init__(self) -> None:
        self.split_ratio = normalize_split_ratio(self.split_ratio)
        total = len(self.partition_data)
        self._bounds = {s: split_bounds(total, s, self.split_ratio) for s in ("train", "val", "test")}
        self._gen = torch.Generator().manual_seed(self.seed)

    @classmethod
    def from_partition_data(cls, data: PartitionData, device: str, rank: int, world_size: int,
                            config: dict[str, Any]) -> "FlareRuntimeLoader":
        chunk_index = data.node_data["c"][0].item().long() if "c" in data.node_data else \
            torch.zeros(data.num_dst_nodes, dtype=torch.long)
        part = data.node_data["partition_id"][0].item() if "partition_id" in data.node_data else None
        pid = int(part[0]) if part is not None and part.numel() else rank
        plan = SnapshotRoutePlan(str(config["graph"]["route"]), str(config["runtime"]["cache"]))
        d = config.get("dtdg", {})
        gl = STGraphLoader.from_partition_data(data, device, chunk_index, rank, world_size,
                                               resident=bool(d.get("resident", True)))
        return cls(partition_id=pid, route_plan=plan,
                   window_state=DTDGWindowState(int(config["model"]["window"]["size"])), partition_data=gl.data,
                   graph_loader=gl, device=device, rank=rank, world_size=world_size, chunk_index=chunk_index,
                   train_chunk_order=d.get("chunk_order"),
                   train_chunk_decay=_parse_chunk_decay(d.get("chunk_decay"), gl.chunk_count),
                   train_num_full_snaps=max(1, int(d.get("num_full_snaps", 1))),
                   split_ratio=config.get("data", {}).get("split_ratio"),
                   window_from_size=bool(d.get("window_from_size", False)),
                   seed=int(config.get("train", {}).get("seed", 0)))

    def load_block(self, index: int):
        return self.graph_loader.fetch_graph(index)

    def load_snapshot(self, index: int, split: str) -> DTDGBatch:
        return _block_to_batch(self.load_block(index), split, self.window_state.window_size, self.route_plan)

    def _publish_row_order(self, perm: torch.Tensor | None) -> None:
        """NVLink halo: tell the peers where this rank's rows are (collective; every
        rank calls it at the same point of the epoch)."""
        from starry_unigraph.parallel.halo import get_halo_context

        hc = get_halo_context()
        if hc is None:
            return
        ids = None
        if perm is not None:
            dst_ids = self.partition_data.dst_ids[0].item().to(perm.device)
            ids = dst_ids[perm.long()]
        hc.set_row_order(ids)

    def iter_train(self, split: str = "train", max_steps: int | None = None) -> Iterable[STGraphBlob]:
        start, end = self._bounds["train"]
        loader = self.graph_loader[start:end]
        order = _parse_chunk_order(self.train_chunk_order, loader.chunk_count, self._gen)
        perm, _ = loader._get_perm_ends(order, self.train_chunk_decay, self.train_num_full_snaps)
        self._publish_row_order(perm)
        window = self.window_state.window_size if self.window_from_size else None
        for i, blob in enumerate(loader(chunk_order=order, chunk_decay=self.train_chunk_decay,
                                        num_full_snaps=self.train_num_full_snaps, window=window)):
            if max_steps is not None and i >= max_steps:
                break
            self.cursor = blob.snapshot_index + 1
            self.window_state.store(blob.snapshot_index)
            yield blob

    def _replay(self, split: str, tag: str) -> Iterable[DTDGBatch]:
        self._publish_row_order(None)  # evaluation reads snapshots in the stored row order
        _, train_end = self._bounds["train"]
        s, e = self._bounds[split]
        for index in range(e):
            batch = self.load_snapshot(index, split)
            batch.chain = "snapshot_warmup" if (index < train_end or index < s) else tag
            self.cursor = index + 1
            yield batch

    def iter_eval(self, split: str = "val") -> Iterable[DTDGBatch]:
        yield from self._replay(split, "snapshot_eval")

    def iter_predict(self, split: str = "test") -> Iterable[DTDGBatch]:
        yield from self._replay(split, "snapshot_predict")

    def build_snapshot_index(self) -> dict[str, Any]:
        return self.graph_loader.build_snapshot_index() | {"window_size": self.window_state.window_size,
                                                          "partition_id": self.partition_id,
                                                          "pipeline": "flare_native"}

    def dump_state(self) -> dict[str, Any]:
        return {"cursor": self.cursor, "partition_id": self.partition_id, "snapshot_count": len(self.partition_data),
                "snapshot_index": self.build_snapshot_index(), "window_state": self.window_state.describe(),
                "route_plan": self.route_plan.describe(), "local_nodes": int(self.partition_data.num_dst_nodes),
                "chunk_count": int(self.chunk_index.max() + 1) if self.chunk_index.numel() else 0}

    def describe_window_state(self) -> dict[str, Any]:
        return self.window_state.describe()

    def describe_route_cache(self) -> dict[str, Any]:
        return self.route_plan.describe() | {
            "partition_id": self.partition_id, "local_nodes": int(self.partition_data.num_dst_nodes),
            "chunk_count": int(self.chunk_index.max() + 1) if self.chunk_index.numel() else 0,
            "loader": "STGraphLoader", "chunk_order": self.train_chunk_order, "chunk_decay": self.train_chunk_decay,
            "num_full_snaps": self.train_num_full_snaps, "window_from_size": self.window_from_size}

    def run_train_step(self, runtime: Any, blob: Any) -> dict[str, Any]:
        from .training import run_flare_train_step

        return run_flare_train_step(runtime, blob, {"meta": {}})

    def run_eval_step(self, runtime: Any, batch: Any) -> dict[str, Any]:
        from .training import run_flare_eval_step

        return run_flare_eval_step(runtime, batch, {"meta": {}})

    def run_predict_step(self, runtime: Any, batch: Any) -> dict[str, Any]:
        from .training import run_flare_predict_step

        return run_flare_predict_step(runtime, batch, {"meta": {}})
