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
                 world_size: int, part_chunks: list[list[tuple[int, int]]] | None = None,
                 part_events: list[list[int]] | None = None):
        """`part_chunks[p]` lists the chunk ids of every rank p and `part_events[p]` their
        event counts (default: this rank's only, for one-rank runs). A chunk runs as
        steps of at most ``train.batch_size`` events in time order; without event counts
        (artifacts written before they were recorded) each chunk is one step."""
        self.chunks = chunks
        self.chunk_manifest = manifest
        self.config = config
        self.device = device
        self.rank = rank
        self.world_size = world_size
        self.cursor = 0
        self._ctdg = None
        self.step_events = max(1, int(config.get("train", {}).get("batch_size", 0) or 1 << 62))
        # within a slice: the preprocessor's dependence-respecting schedule when recorded
        rank_of = {tuple(cid): i for i, cid in enumerate(manifest.get("order", []))}
        mine = sorted(chunks.chunks, key=lambda c: (c.chunk_id[0], rank_of.get(tuple(c.chunk_id), len(rank_of)),
                                                     c.chunk_id[1]))
        counted = part_events is not None or part_chunks is None
        if part_chunks is None:
            part_chunks = [[tuple(c.chunk_id) for c in chunks.chunks]]
            part_events = [[c.num_events for c in chunks.chunks]]
        if not counted:
            part_events = [[1] * len(p) for p in part_chunks]
        size = self.step_events if counted else 1 << 62

        def pieces(n: int) -> int:
            return max(1, -(-int(n) // size))

        slices = sorted({int(cid[0]) for part in part_chunks for cid in part})
        steps_in = {t: max(sum(pieces(n) for cid, n in zip(part, ev) if int(cid[0]) == t)
                           for part, ev in zip(part_chunks, part_events)) for t in slices}
        ratio = normalize_split_ratio(config.get("data", {}).get("split_ratio"))
        self._splits: dict[str, list[Any]] = {}
        for split in ("train", "val", "test"):
            units: list[Any] = []
            for t in slices[slice(*split_bounds(len(slices), split, ratio))] if slices else []:
                own = []
                for c in (c for c in mine if c.chunk_id[0] == t):
                    n = c.num_events
                    own.extend((c, lo, min(n, lo + size)) for lo in range(0, max(n, 1), size))
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
        parts = [json.loads((clusters / f"part_{p:03d}" / "cluster_manifest.json").read_text())
                 for p in range(world_size)]
        part_chunks = [[tuple(cid) for cid in m["chunks"]] for m in parts]
        part_events = [m["chunk_events"] for m in parts] if all("chunk_events" in m for m in parts) else None
        return cls(chunks, manifest, config, device, rank, world_size, part_chunks, part_events)

    def attach_ctdg(self, online_runtime: Any) -> None:
        self._ctdg = online_runtime

    def _batch(self, unit, split: str) -> CTDGDataBatch:
        """The step of `unit`: (chunk, first event, end event), or None for a padding step
        that takes part in the step's collectives with no events."""
        ds = self._ctdg.dataset
        if unit is None:
            none = torch.zeros(0, dtype=torch.long)
            return CTDGDataBatch(index=-1, split=split, event_ids=none, src=none, dst=none, ts=torch.zeros(0),
                                 edge_feat=ds.edge_feat[none])
        chunk, lo, hi = unit if isinstance(unit, tuple) else (unit, 0, unit.num_events)
        ev = chunk.events
        eid = ev["eid"][lo:hi]
        return CTDGDataBatch(index=chunk.chunk_id[0], split=split, event_ids=eid, src=ev["src"][lo:hi],
                             dst=ev["dst"][lo:hi], ts=ev["ts"][lo:hi], edge_feat=ds.edge_feat[eid])

    def iter_chunks(self, split: str) -> Iterable[Any]:
        """This rank's chunks of the split, each once (without the padding steps)."""
        last = None
        for u in self._splits["test" if split == "predict" else split]:
            if u is not None and u[0] is not last:
                last = u[0]
                yield last

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
