"""Chunk generation entry point (reference backends/chunk/prepare/generate_chunk.py,
broken there): chunks plus their dependence routes and a run order."""
from __future__ import annotations

from typing import Any

from .adaptive import ChunkGenerator, schedule


def generate_chunks(src, dst, ts, num_nodes: int, num_clusters: int = 8, time_slices: int = 16,
                    adaptive: bool = False, seed: int = 0, with_routes: bool = False) -> Any:
    """Chunks of the stream (a list), or with ``with_routes`` a dict with the
    chunks, their dependence routes, the cluster map and a dependency-respecting
    run order."""
    gen = ChunkGenerator(num_clusters=num_clusters, time_slices=time_slices, adaptive=adaptive, seed=seed)
    out = gen.generate(src, dst, ts, num_nodes)
    if not with_routes:
        return out["chunks"]
    out["order"] = schedule(out["routes"])
    return out
