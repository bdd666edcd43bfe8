"""Chunk runtime loader (reference runtime/chunk/session_loader.py:20-139, stubs there).

Iterates this rank's chunks slice by slice; each chunk's events form one
training step of the CTDG online runtime (memory, mailbox, temporal attention,
fused sm_100a step on CUDA), so chunk mode trains the same TGN-family models
in time-slice x cluster units.

Ranks run in lock step: the train / validation / test splits are ranges of the
global time slices (the same on every rank, so no rank trains on a slice that
another evaluates), and within a slice every rank takes as many steps as the
rank with the most chunks in it, padding with empty steps. Every step of the
CTDG runtime takes part in the same collectives (gradient all-reduce, memory
and mail exchanges), so equal step counts keep them matched, and memory pushed
in slice t lands before any rank reads it in slice t + 1.
"""
from __future__ import annotations

from pathlib import Path
from typing import Any, Iterable

import torch

from starry_unigraph.backends.ctdg.runtime.data import CTDGDataBatch
from starry_unigraph.data.chunk_data import ChunkData
from starry_unigraph.runtime._split import normalize_split_ratio, split_bounds


class ChunkRuntimeLoader:
    def __init__(self, chunks: ChunkData, manifest: dict[str, Any], config: dict[str, Any], device: str, rank: int,
                 world_size: int, part_chunks: list[list[tuple[int, int]]] | None = None):
        """`part_chunks[p]` lists the chunk ids of every rank p (default: this rank's
        only, for one-rank runs)."""
        self.chunks = chunks
        self.chunk_manifest = manifest
        self.config = config
        self.device = device
        self.rank = rank
        self.world_size = world_size
        self.cursor = 0
        self._ctdg = None
        # within a slice: the preprocessor's dependence-respecting schedule when recorded
        rank_of = {tuple(cid): i for i, cid in enumerate(manifest.get("order", []))}
        mine = sorted(chunks.chunks, key=lambda c: (c.chunk_id[0], rank_of.get(tuple(c.chunk_id), len(rank_of)),
                                                     c.chunk_id[1]))
        parts = part_chunks if part_chunks is not None else [[tuple(c.chunk_id) for c in chunks.chunks]]
        slices = sorted({int(cid[0]) for part in parts for cid in part})
        steps_in = {t: max(sum(1 for cid in part if int(cid[0]) == t) for part in parts) for t in slices}
        ratio = normalize_split_ratio(config.get("data", {}).get("split_ratio"))
        self._splits: dict[str, list[Any]] = {}
        for split in ("train", "val", "test"):
            units: list[Any] = []
            for t in slices[slice(*split_bounds(len(slices), split, ratio))] if slices else []:
                own = [c for c in mine if c.chunk_id[0] == t]
                units.extend(own + [None] * (steps_in[t] - len(own)))  # None: an empty step
            self._splits[split] = units

    @classmethod
    def from_prepared_artifacts(cls, prepared_dir: Path, device: str, rank: int, world_size: int,
                                config: dict[str, Any]) -> "ChunkRuntimeLoader":
        import json

        clusters = Path(prepared_dir) / "clusters"
        part = clusters / f"part_{min(rank, world_size - 1):03d}"
        chunks = ChunkData.load(part / "chunks.pt")
        manifest = json.loads((part / "cluster_manifest.json").read_text())
        routes_path = Path(prepared_dir) / "routes" / "manifest.json"
        if routes_path.exists():
            manifest["order"] = json.loads(routes_path.read_text()).get("order", [])
        part_chunks = [[tuple(cid) for cid in json.loads((clusters / f"part_{p:03d}" / "cluster_manifest.json")
                                                          .read_text())["chunks"]] for p in range(world_size)]
        return cls(chunks, manifest, config, device, rank, world_size, part_chunks)

    def attach_ctdg(self, online_runtime: Any) -> None:
        self._ctdg = online_runtime

    def _batch(self, chunk, split: str) -> CTDGDataBatch:
        ds = self._ctdg.dataset
        if chunk is None:  # padding step: takes part in the step's collectives with no events
            none = torch.zeros(0, dtype=torch.long)
            return CTDGDataBatch(index=-1, split=split, event_ids=none, src=none, dst=none, ts=torch.zeros(0),
                                 edge_feat=ds.edge_feat[none])
        ev = chunk.events
        return CTDGDataBatch(index=chunk.chunk_id[0], split=split, event_ids=ev["eid"], src=ev["src"], dst=ev["dst"],
                             ts=ev["ts"], edge_feat=ds.edge_feat[ev["eid"]])

    def iter_chunks(self, split: str) -> Iterable[Any]:
        """This rank's chunks of the split (without the padding steps)."""
        yield from (c for c in self._splits["test" if split == "predict" else split] if c is not None)

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
