"""Chunk = time slice x node cluster, the atomic unit of the chunk pipeline
(reference data/chunk_atomic.py:19-111, where materialisation is a stub).

A chunk holds its events in a temporal CSR over the cluster's master nodes
(L1), the cross-cluster neighbours with their home clusters (L2) and
scheduling metadata (L3). ``materialize`` samples the most recent neighbours of
each event endpoint from the chunk's T-CSR and returns the local message-flow
block plus the manifest of remote rows that must be fetched from other ranks;
``complete`` assembles the neighbours' feature rows from the local feature store
and the fetched remote rows.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any, Callable

import torch
from torch import Tensor


@dataclass
class RemoteManifest:
    remote_node_ids: Tensor   # [N_remote] global ids to fetch
    remote_owners: Tensor     # [N_remote] owning rank
    local_slots: Tensor       # [N_remote] slot in the materialised block


@dataclass
class SpatialDeps:
    """Same-time-slice communication with other clusters."""
    peer_clusters: Tensor     # [P]
    send_counts: Tensor       # [P]


@dataclass
class StateDeps:
    """State read/write dependencies across time slices."""
    read_from: Tensor         # [R] chunk ids whose state is read
    write_nodes: Tensor       # [W] nodes whose state this chunk writes


@dataclass
class ChunkAtomic:
    chunk_id: tuple[int, int]
    time_range: tuple[float, float]
    node_set: Tensor
    tcsr_rowptr: Tensor
    tcsr_col: Tensor
    tcsr_ts: Tensor
    tcsr_edge_id: Tensor
    cross_node_ids: Tensor
    cross_node_home: Tensor
    cross_edge_count: Tensor
    load_estimate: float = 0.0
    spatial_deps: SpatialDeps | None = None
    state_deps: StateDeps | None = None
    events: dict[str, Tensor] | None = None   # src, dst, ts, eid of the chunk's events
    _neg_hook: Callable | None = field(default=None, repr=False, compare=False)
    _neighbor_hook: Callable | None = field(default=None, repr=False, compare=False)

    def register_negative_hook(self, fn: Callable) -> None:
        self._neg_hook = fn

    def register_neighbor_hook(self, fn: Callable) -> None:
        self._neighbor_hook = fn

    @property
    def num_events(self) -> int:
        return 0 if self.events is None else int(self.events["src"].numel())

    def materialize(self, sampler_cfg: Any, owner: Tensor | None = None, rank: int = 0):
        """Phase 1: local temporal sampling for every event endpoint of the chunk,
        plus the manifest of neighbours owned by other ranks."""
        from starry_unigraph.backends.ctdg.runtime.models import DenseBlock
        from starry_unigraph.backends.ctdg.runtime.sampler import TemporalCSR

        from .batch_data import BatchData

        k = int((getattr(sampler_cfg, "num_neighbors", None) or [10])[0])
        ev = self.events or {"src": torch.zeros(0, dtype=torch.long), "dst": torch.zeros(0, dtype=torch.long),
                             "ts": torch.zeros(0), "eid": torch.zeros(0, dtype=torch.long)}
        roots = torch.unique(torch.cat([ev["src"], ev["dst"]]))
        if self._neighbor_hook is not None:
            block = self._neighbor_hook(roots, ev)
        else:
            # chunk-local T-CSR over global ids of the master nodes
            n_glob = int(max(int(self.node_set.max()) + 1 if self.node_set.numel() else 0,
                             int(roots.max()) + 1 if roots.numel() else 0))
            rowptr = torch.zeros(n_glob + 1, dtype=torch.long)
            deg = self.tcsr_rowptr[1:] - self.tcsr_rowptr[:-1]
            counts = torch.zeros(n_glob, dtype=torch.long)
            counts[self.node_set] = deg
            rowptr[1:] = torch.cumsum(counts, 0)
            csr = TemporalCSR(rowptr, self.tcsr_col, self.tcsr_edge_id, self.tcsr_ts.long(), n_glob)
            rts = torch.full((roots.numel(),), int(ev["ts"].max()) if ev["ts"].numel() else 0, dtype=torch.long)
            block = csr.sample_torch(roots, rts, k)
        neg = self._neg_hook(ev) if self._neg_hook is not None else None
        nbr = block.nbr[block.mask()] if isinstance(block, DenseBlock) else torch.zeros(0, dtype=torch.long)
        if owner is not None and nbr.numel():
            remote = owner[nbr] != rank
            ids = torch.unique(nbr[remote])
            manifest = RemoteManifest(ids, owner[ids], torch.arange(ids.numel()))
        else:
            manifest = RemoteManifest(torch.zeros(0, dtype=torch.long), torch.zeros(0, dtype=torch.long),
                                      torch.zeros(0, dtype=torch.long))
        batch = BatchData(mfg=block, node_ids=roots, pos_src=ev["src"], pos_dst=ev["dst"],
                          neg_src=ev["src"] if neg is not None else None, neg_dst=neg, timestamps=ev["ts"],
                          chunk_id=self.chunk_id, remote_manifest={"count": int(manifest.remote_node_ids.numel())})
        return batch, manifest

    def complete(self, local_mfg: Any, remote_data: dict[str, Tensor] | None = None, local_store: Any = None,
                 feat_name: str = "x") -> Any:
        """Phase 2: the feature rows of every sampled neighbour slot, in the block's
        [roots, k] layout (zero rows for empty slots), into ``batch.nbr_feat``.

        Rows of nodes listed in ``remote_data`` (``{"node_ids": [R], "rows": [R, F]}``,
        the answer to the phase-1 manifest) come from it; every other neighbour is
        read from ``local_store`` (a ``FeatureStore`` of the rows this rank owns).
        ``batch.local_node_mask`` marks the slots served locally. Without a store the
        batch is returned as it is."""
        block = getattr(local_mfg, "mfg", None)
        if local_store is None or block is None or not hasattr(block, "nbr"):
            return local_mfg
        nbr = block.nbr
        valid = block.mask()
        flat = nbr[valid]
        is_remote = torch.zeros(flat.numel(), dtype=torch.bool)
        rows = None
        if remote_data and remote_data.get("node_ids") is not None and remote_data["node_ids"].numel():
            key, order = torch.sort(remote_data["node_ids"].long())
            pos = torch.searchsorted(key, flat).clamp(max=key.numel() - 1)
            is_remote = key[pos] == flat
            remote_rows = remote_data["rows"][order[pos[is_remote]]]
            rows = torch.zeros(flat.numel(), remote_rows.size(1), dtype=remote_rows.dtype)
            rows[is_remote] = remote_rows
        local_rows = local_store.get_node_feat(flat[~is_remote], feat_name) if bool((~is_remote).any()) else None
        width = local_store.feat_dim(feat_name)
        if rows is None:
            dtype = local_rows.dtype if local_rows is not None else torch.float32
            rows = torch.zeros(flat.numel(), width, dtype=dtype)
        if local_rows is not None:
            rows[~is_remote] = local_rows.to(rows)
        out = torch.zeros(*nbr.shape, width, dtype=rows.dtype)
        out[valid] = rows
        local_mask = torch.zeros(nbr.shape, dtype=torch.bool)
        local_mask[valid] = ~is_remote
        local_mfg.nbr_feat = out
        local_mfg.local_node_mask = local_mask
        local_mfg.remote_manifest = dict(local_mfg.remote_manifest or {}) | {"filled": int(is_remote.sum())}
        return local_mfg
