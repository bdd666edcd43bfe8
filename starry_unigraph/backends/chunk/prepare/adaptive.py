"""Chunk generation: time slices x node clusters with dependence routes
(reference design: backends/chunk/prepare/adaptive.py:293-484, which does not
parse there).

* Clusters: the native partitioner on the lifetime graph. With
  ``adaptive=True`` the cluster count grows when too many events cross
  clusters: if the cross-cluster fraction r exceeds ``info_loss_threshold``
  the count becomes ceil(n * r / threshold) and the partition is redone (once,
  capped at ``max_clusters``), the reference's rule.
* Temporal dependence: a chunk (slice t, cluster c) depends on the chunks of
  cluster c in earlier slices, newest first, weighted decay_base^k for the
  k-th one back (k = 1, 2, ...).
* Spatial (GNN) dependence: in one slice, chunk (t, c) depends on chunk
  (t, c') when an event of slice t joins a node of c and a node of c' (either
  direction). The reference tests this on the chunks' own edge lists, which
  keep only intra-cluster edges, so it can never fire; here the slice's
  events are used.
* Negatives: ``neg_per_event`` destinations per event drawn from the stream's
  destination pool.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Any

import torch

from starry_unigraph.data.chunk_builder import ChunkBuilder


@dataclass
class DependenceRoute:
    chunk_id: tuple[int, int]
    temporal_deps: list[tuple[int, int]] = field(default_factory=list)  # newest first
    gnn_deps: list[tuple[int, int]] = field(default_factory=list)
    decay_weights: torch.Tensor = field(default_factory=lambda: torch.zeros(0))

    def describe(self) -> dict[str, Any]:
        return {"chunk": list(self.chunk_id), "temporal": [list(d) for d in self.temporal_deps],
                "gnn": [list(d) for d in self.gnn_deps], "decay": [round(float(w), 6) for w in self.decay_weights]}


def cross_cluster_ratio(src: torch.Tensor, dst: torch.Tensor, cluster: torch.Tensor) -> float:
    if src.numel() == 0:
        return 0.0
    return float((cluster[src.long()] != cluster[dst.long()]).float().mean())


class ChunkGenerator:
    def __init__(self, num_clusters: int | None = None, time_slices: int = 16, adaptive: bool = True,
                 nodes_per_cluster: int = 100_000, seed: int = 0, info_loss_threshold: float = 0.3,
                 max_clusters: int = 1024, decay_base: float = 0.9, edge_share: float = 0.9):
        self.edge_share = float(edge_share)  # cluster balance: see ChunkBuilder
        self.num_clusters = num_clusters
        self.time_slices = time_slices
        self.adaptive = adaptive
        self.nodes_per_cluster = nodes_per_cluster
        self.seed = seed
        self.info_loss_threshold = float(info_loss_threshold)
        self.max_clusters = int(max_clusters)
        self.decay_base = float(decay_base)

    def cluster_count(self, num_nodes: int) -> int:
        return self.num_clusters or max(1, (num_nodes + self.nodes_per_cluster - 1) // self.nodes_per_cluster)

    def generate_graph_clusters(self, src: torch.Tensor, dst: torch.Tensor, num_nodes: int,
                                num_clusters: int | None = None) -> tuple[torch.Tensor, int, float]:
        """(cluster of every node, cluster count, cross-cluster event fraction)."""
        n = num_clusters or self.cluster_count(num_nodes)
        cluster = ChunkBuilder(num_clusters=n, seed=self.seed, edge_share=self.edge_share).clusters(
            src.long(), dst.long(), num_nodes)
        ratio = cross_cluster_ratio(src, dst, cluster)
        if self.adaptive and ratio > self.info_loss_threshold and n < self.max_clusters:
            n = min(self.max_clusters, max(n + 1, math.ceil(n * ratio / self.info_loss_threshold)))
            cluster = ChunkBuilder(num_clusters=n, seed=self.seed, edge_share=self.edge_share).clusters(
                src.long(), dst.long(), num_nodes)
            ratio = cross_cluster_ratio(src, dst, cluster)
        return cluster, n, ratio

    def build_routes(self, chunk_ids: list[tuple[int, int]], src: torch.Tensor, dst: torch.Tensor,
                     slice_of_event: torch.Tensor, cluster: torch.Tensor) -> list[DependenceRoute]:
        present = set(chunk_ids)
        by_cluster: dict[int, list[int]] = {}
        for t, c in chunk_ids:
            by_cluster.setdefault(c, []).append(t)
        # (slice, cluster a, cluster b) for every cross-cluster event, both directions
        ca, cb = cluster[src.long()], cluster[dst.long()]
        cross = ca != cb
        pairs = torch.stack([slice_of_event[cross].long(), ca[cross], cb[cross]], dim=1)
        pairs = torch.unique(torch.cat([pairs, pairs[:, [0, 2, 1]]]), dim=0)
        spatial: dict[tuple[int, int], list[tuple[int, int]]] = {}
        for t, a, b in pairs.tolist():
            if (t, a) in present and (t, b) in present:
                spatial.setdefault((t, a), []).append((t, b))
        routes = []
        for t, c in chunk_ids:
            earlier = sorted((s for s in by_cluster[c] if s < t), reverse=True)
            k = torch.arange(1, len(earlier) + 1, dtype=torch.float32)
            routes.append(DependenceRoute(chunk_id=(t, c), temporal_deps=[(s, c) for s in earlier],
                                          gnn_deps=sorted(spatial.get((t, c), [])),
                                          decay_weights=self.decay_base ** k))
        return routes

    def generate(self, src, dst, ts, num_nodes: int, neg_per_event: int = 1, eid=None) -> dict[str, Any]:
        src, dst = src.long(), dst.long()
        cluster, n_clusters, ratio = self.generate_graph_clusters(src, dst, num_nodes)
        builder = ChunkBuilder(n_clusters, self.time_slices, self.adaptive, seed=self.seed, edge_share=self.edge_share)
        slice_of_event = builder.slice_ids(src, dst, ts)
        chunks = builder.build(src, dst, ts, num_nodes, eid=eid, slice_ids=slice_of_event, clusters=cluster)
        g = torch.Generator().manual_seed(self.seed)
        pool = torch.unique(dst)
        for ch in chunks:
            ch.events["neg"] = pool[torch.randint(0, pool.numel(), (ch.num_events * neg_per_event,), generator=g)]
        routes = self.build_routes([c.chunk_id for c in chunks], src, dst, slice_of_event, cluster)
        load = torch.bincount(cluster[src], minlength=n_clusters).float() if src.numel() else torch.zeros(n_clusters)
        return {"chunks": chunks, "routes": routes, "clusters": cluster, "num_clusters": n_clusters,
                "cross_ratio": ratio, "builder": builder.describe() | {
                    "events_max_over_mean": round(float(load.max() / load.mean().clamp_min(1e-9)), 4)}}


def schedule(routes: list[DependenceRoute]) -> list[tuple[int, int]]:
    """Chunk order in which every chunk runs after its temporal dependencies
    (Kahn's algorithm; ties broken by (slice, cluster))."""
    import heapq

    deps = {r.chunk_id: {d for d in r.temporal_deps} for r in routes}
    users: dict[tuple[int, int], list[tuple[int, int]]] = {}
    for cid, ds in deps.items():
        for d in ds:
            users.setdefault(d, []).append(cid)
    waiting = {cid: len([d for d in ds if d in deps]) for cid, ds in deps.items()}
    ready = [cid for cid, n in waiting.items() if n == 0]
    heapq.heapify(ready)
    order = []
    while ready:
        cid = heapq.heappop(ready)
        order.append(cid)
        for u in users.get(cid, []):
            waiting[u] -= 1
            if waiting[u] == 0:
                heapq.heappush(ready, u)
    if len(order) != len(deps):
        raise ValueError("dependence routes contain a cycle")
    return order
