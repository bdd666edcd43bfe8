"""Build chunks (time slice x node cluster) from an event stream
(reference data/chunk_builder.py:21-92, a stub there).

Time slices come from the native adaptive split (staleness-driven) or equal
counts; node clusters from the native partitioner on the lifetime graph. Each
chunk keeps the events whose source lies in the cluster, a T-CSR of the
cluster's incoming events and its cross-cluster neighbours.
"""
from __future__ import annotations

from typing import Any

import torch

from .chunk_atomic import ChunkAtomic, SpatialDeps, StateDeps


class ChunkBuilder:
    def __init__(self, num_clusters: int = 8, time_slices: int = 16, adaptive: bool = False,
                 base_batch_size: int = 1000, graph_feature: float = 0.5, seed: int = 0, edge_share: float = 0.9):
        """`edge_share`: share of the partitioner's vertex weight put on event endpoints (the
        rest on nodes), so clusters carry similar event counts: a chunk's step costs its
        events, and on a skewed stream node-balanced clusters leave most events in one."""
        self.edge_share = float(edge_share)
        self.num_clusters = max(1, int(num_clusters))
        self.time_slices = max(1, int(time_slices))
        self.adaptive = adaptive
        self.base_batch_size = base_batch_size
        self.graph_feature = graph_feature
        self.seed = seed

    def slice_ids(self, src, dst, ts) -> torch.Tensor:
        n = src.numel()
        if self.adaptive:
            from starry_unigraph.ops import native_ext

            nat = native_ext()
            if nat is not None:
                return nat.adaptive_split(src.long(), dst.long(), ts.double(), self.base_batch_size,
                                          self.graph_feature).group_index
        per = max(1, (n + self.time_slices - 1) // self.time_slices)
        return torch.arange(n) // per

    def clusters(self, src, dst, num_nodes: int) -> torch.Tensor:
        from starry_unigraph.backends.dtdg.dtdg_prepare import apply_partition

        return apply_partition(torch.stack([src, dst]), num_nodes, self.num_clusters, self.seed,
                               edge_share=self.edge_share)

    def build(self, src, dst, ts, num_nodes: int, eid=None, slice_ids=None, clusters=None) -> list[ChunkAtomic]:
        """Chunks of the stream; `slice_ids` (per event) and `clusters` (per node)
        may be given precomputed, else they come from slice_ids() / clusters()."""
        eid = torch.arange(src.numel()) if eid is None else eid
        sl = self.slice_ids(src, dst, ts) if slice_ids is None else slice_ids
        cl = self.clusters(src, dst, num_nodes) if clusters is None else clusters
        if clusters is not None:
            self.num_clusters = max(self.num_clusters, int(cl.max()) + 1 if cl.numel() else 1)
        out: list[ChunkAtomic] = []
        for t in range(int(sl.max()) + 1 if sl.numel() else 0):
            in_t = sl == t
            for c in range(self.num_clusters):
                m = in_t & (cl[src] == c)
                if not bool(m.any()):
                    continue
                s, d, tt, e = src[m], dst[m], ts[m], eid[m]
                nodes = torch.nonzero(cl == c).view(-1)
                loc = torch.full((num_nodes,), -1, dtype=torch.long)
                loc[nodes] = torch.arange(nodes.numel())
                into = loc[d] >= 0
                order = torch.argsort(loc[d[into]], stable=True)
                counts = torch.bincount(loc[d[into]], minlength=nodes.numel())
                rowptr = torch.zeros(nodes.numel() + 1, dtype=torch.long)
                rowptr[1:] = torch.cumsum(counts, 0)
                cross = torch.unique(torch.cat([s, d])[cl[torch.cat([s, d])] != c])
                home = cl[cross]
                out.append(ChunkAtomic(
                    chunk_id=(t, c), time_range=(float(tt.min()), float(tt.max())), node_set=nodes,
                    tcsr_rowptr=rowptr, tcsr_col=s[into][order], tcsr_ts=tt[into][order].long(),
                    tcsr_edge_id=e[into][order], cross_node_ids=cross, cross_node_home=home,
                    cross_edge_count=torch.bincount(home, minlength=self.num_clusters),
                    load_estimate=float(m.sum()),
                    spatial_deps=SpatialDeps(torch.unique(home), torch.bincount(home, minlength=self.num_clusters)),
                    state_deps=StateDeps(torch.tensor([t - 1]) if t > 0 else torch.zeros(0, dtype=torch.long),
                                         torch.unique(torch.cat([s, d]))),
                    events={"src": s, "dst": d, "ts": tt, "eid": e}))
        return out

    def describe(self) -> dict[str, Any]:
        return {"num_clusters": self.num_clusters, "time_slices": self.time_slices, "adaptive": self.adaptive,
                "edge_share": self.edge_share}
