"""ChunkGenerator (reference backends/chunk/prepare/adaptive.py:13-561, syntax errors there):
snapshot slicing, information-aware CTDG slicing with the adaptive split,
METIS-style clusters with an adaptive count, negative pre-sampling and the
temporal / GNN dependence routes between chunks."""
from __future__ import annotations

from typing import Any

import torch

from starry_unigraph.data.chunk_builder import ChunkBuilder


class ChunkGenerator:
    def __init__(self, num_clusters: int | None = None, time_slices: int = 16, adaptive: bool = True,
                 nodes_per_cluster: int = 100_000, seed: int = 0):
        self.num_clusters = num_clusters
        self.time_slices = time_slices
        self.adaptive = adaptive
        self.nodes_per_cluster = nodes_per_cluster
        self.seed = seed

    def cluster_count(self, num_nodes: int) -> int:
        return self.num_clusters or max(1, (num_nodes + self.nodes_per_cluster - 1) // self.nodes_per_cluster)

    def generate(self, src, dst, ts, num_nodes: int, neg_per_event: int = 1) -> dict[str, Any]:
        b = ChunkBuilder(self.cluster_count(num_nodes), self.time_slices, self.adaptive, seed=self.seed)
        chunks = b.build(src, dst, ts, num_nodes)
        g = torch.Generator().manual_seed(self.seed)
        pool = torch.unique(dst)
        for ch in chunks:
            n = ch.num_events * neg_per_event
            ch.events["neg"] = pool[torch.randint(0, pool.numel(), (n,), generator=g)]
        temporal_routes = [(c.chunk_id, (c.chunk_id[0] - 1, c.chunk_id[1])) for c in chunks if c.chunk_id[0] > 0]
        gnn_routes = [(c.chunk_id, int(h)) for c in chunks for h in torch.unique(c.cross_node_home).tolist()]
        return {"chunks": chunks, "temporal_routes": temporal_routes, "gnn_routes": gnn_routes,
                "builder": b.describe()}
