"""Chunk runtime loader (reference runtime/chunk/session_loader.py:20-139, stubs there).

Iterates this rank's chunks in time-slice order; each chunk's events form one
training step of the CTDG online runtime (memory, mailbox, temporal attention,
fused sm_100a step on CUDA), so chunk mode trains the same TGN-family models
in time-slice x cluster units."""
from __future__ import annotations

from pathlib import Path
from typing import Any, Iterable

import torch

from starry_unigraph.backends.ctdg.runtime.data import CTDGDataBatch
from starry_unigraph.data.chunk_data import ChunkData
from starry_unigraph.runtime._split import normalize_split_ratio, split_bounds


class ChunkRuntimeLoader:
    def __init__(self, chunks: ChunkData, manifest: dict[str, Any], config: dict[str, Any], device: str, rank: int,
                 world_size: int):
        self.chunks = chunks
        self.chunk_manifest = manifest
        self.config = config
        self.device = device
        self.rank = rank
        self.world_size = world_size
        self.cursor = 0
        self._ctdg = None
        # run order: the preprocessor's dependency-respecting schedule when recorded
        # (every chunk after the chunks of its cluster in earlier slices), else by (slice, cluster)
        rank_of = {tuple(cid): i for i, cid in enumerate(manifest.get("order", []))}
        ordered = sorted(chunks.chunks, key=lambda c: (rank_of.get(tuple(c.chunk_id), len(rank_of)),
                                                       c.chunk_id[0], c.chunk_id[1]))
        ratio = normalize_split_ratio(config.get("data", {}).get("split_ratio"))
        n = len(ordered)
        self._splits = {s: ordered[slice(*split_bounds(n, s, ratio))] for s in ("train", "val", "test")}

    @classmethod
    def from_prepared_artifacts(cls, prepared_dir: Path, device: str, rank: int, world_size: int,
                                config: dict[str, Any]) -> "ChunkRuntimeLoader":
        import json

        part = Path(prepared_dir) / "clusters" / f"part_{min(rank, world_size - 1):03d}"
        chunks = ChunkData.load(part / "chunks.pt")
        manifest = json.loads((part / "cluster_manifest.json").read_text())
        routes_path = Path(prepared_dir) / "routes" / "manifest.json"
        if routes_path.exists():
            manifest["order"] = json.loads(routes_path.read_text()).get("order", [])
        return cls(chunks, manifest, config, device, rank, world_size)

    def attach_ctdg(self, online_runtime: Any) -> None:
        self._ctdg = online_runtime

    def _batch(self, chunk, split: str) -> CTDGDataBatch:
        ev = chunk.events
        ds = self._ctdg.dataset
        return CTDGDataBatch(index=chunk.chunk_id[0], split=split, event_ids=ev["eid"], src=ev["src"], dst=ev["dst"],
                             ts=ev["ts"], edge_feat=ds.edge_feat[ev["eid"]])

    def iter_chunks(self, split: str) -> Iterable[Any]:
        yield from self._splits["test" if split == "predict" else split]

    def iter_train(self, split: str = "train") -> Iterable[CTDGDataBatch]:
        for ch in self._splits["train"]:
            self.cursor += 1
            yield self._batch(ch, "train")

    def iter_eval(self, split: str = "val") -> Iterable[CTDGDataBatch]:
        for ch in self._splits[split]:
            yield self._batch(ch, split)

    def iter_predict(self, split: str = "test") -> Iterable[CTDGDataBatch]:
        yield from self.iter_eval(split)

    def run_train_step(self, runtime: Any, batch: CTDGDataBatch) -> dict[str, Any]:
        return self._ctdg.train_step(batch)

    def run_eval_step(self, runtime: Any, batch: CTDGDataBatch) -> dict[str, Any]:
        return self._ctdg.eval_step(batch, batch.split)

    def run_predict_step(self, runtime: Any, batch: CTDGDataBatch) -> dict[str, Any]:
        return self._ctdg.predict_step(batch)

    def describe_window_state(self) -> dict[str, Any]:
        return {"chunks": len(self.chunks), "cursor": self.cursor}

    def dump_state(self) -> dict[str, Any]:
        return {"cursor": self.cursor, "rank": self.rank, "splits": {k: len(v) for k, v in self._splits.items()}}

    def describe_route_cache(self) -> dict[str, Any]:
        return {"loader": "ChunkRuntimeLoader", **self.chunk_manifest}
