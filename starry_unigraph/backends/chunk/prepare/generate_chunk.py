"""Chunk generation entry point (reference backends/chunk/prepare/generate_chunk.py, broken there)."""
from __future__ import annotations

from starry_unigraph.data.chunk_builder import ChunkBuilder


def generate_chunks(src, dst, ts, num_nodes: int, num_clusters: int = 8, time_slices: int = 16,
                    adaptive: bool = False):
    return ChunkBuilder(num_clusters=num_clusters, time_slices=time_slices, adaptive=adaptive).build(
        src, dst, ts, num_nodes)
