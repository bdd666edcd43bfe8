"""Whole-graph compressed sparse rows (reference data/global_csr.py:15-76, a
protocol only there).

``GlobalCSR`` is the reference's interface: node / edge counts, ``rowptr`` and
``col``, the concatenated neighbours (and edge ids) of a node list, the induced
subgraph of a node list with ids renumbered to [0, N), and ``load`` from a data
root with optional sharding by rank. ``TemporalGlobalCSR`` implements it over an
event stream with rows keyed by destination (the temporal sampler's convention:
a node's neighbours are the sources of events into it, kept in time order), and
adds the temporal reads the chunk builder needs: the neighbours of one node
strictly before a time and a time-window slice.
"""
from __future__ import annotations

from pathlib import Path
from typing import Protocol

import torch
from torch import Tensor


class GlobalCSR(Protocol):
    @property
    def num_nodes(self) -> int: ...

    @property
    def num_edges(self) -> int: ...

    def rowptr(self) -> Tensor: ...

    def col(self) -> Tensor: ...

    def neighbors(self, node_ids: Tensor) -> tuple[Tensor, Tensor]: ...

    def subgraph(self, node_ids: Tensor) -> "GlobalCSR": ...


class TemporalGlobalCSR:
    def __init__(self, src: Tensor, dst: Tensor, ts: Tensor, num_nodes: int, eid: Tensor | None = None):
        from starry_unigraph.backends.ctdg.runtime.sampler import TemporalCSR

        self.src, self.dst, self.ts = src.long(), dst.long(), ts
        self.eid = torch.arange(src.numel()) if eid is None else eid.long()
        self._num_nodes = int(num_nodes)
        self.csr = TemporalCSR.build(self.src, self.dst, self.eid, ts.long(), self._num_nodes)

    # ------------------------------------------------------------------ the protocol
    @property
    def num_nodes(self) -> int:
        return self._num_nodes

    @property
    def num_edges(self) -> int:
        return int(self.csr.nbr.numel())

    def rowptr(self) -> Tensor:
        return self.csr.rowptr

    def col(self) -> Tensor:
        return self.csr.nbr

    def neighbors(self, node_ids: Tensor | int) -> tuple[Tensor, Tensor]:
        """(neighbour ids, edge ids) of every listed node, concatenated in list order,
        each node's run in time order."""
        ids = torch.as_tensor(node_ids).long().view(-1)
        lo, hi = self.csr.rowptr[ids], self.csr.rowptr[ids + 1]
        counts = hi - lo
        if int(counts.sum()) == 0:
            empty = torch.empty(0, dtype=torch.long)
            return empty, empty.clone()
        start = torch.repeat_interleave(lo - (torch.cumsum(counts, 0) - counts), counts)
        pos = start + torch.arange(int(counts.sum()))
        return self.csr.nbr[pos], self.csr.eid[pos]

    def subgraph(self, node_ids: Tensor) -> "TemporalGlobalCSR":
        """Events with both endpoints in `node_ids`, ids renumbered to positions in
        `node_ids` (which need not be sorted); edge ids are kept."""
        ids = node_ids.long().view(-1)
        local = torch.full((self._num_nodes,), -1, dtype=torch.long)
        local[ids] = torch.arange(ids.numel())
        keep = (local[self.src] >= 0) & (local[self.dst] >= 0)
        return TemporalGlobalCSR(local[self.src[keep]], local[self.dst[keep]], self.ts[keep], ids.numel(),
                                 self.eid[keep])

    @classmethod
    def load(cls, data_root: str | Path, rank: int = 0, world_size: int = 1,
             config: dict | None = None) -> "TemporalGlobalCSR":
        """The event stream of the dataset directory `data_root` (any format the raw
        loader reads); with world_size > 1 only rows of the nodes this rank owns under
        the hash partition (node % world_size == rank) are kept."""
        from starry_unigraph.data.raw_temporal import load_raw_temporal_events

        root = Path(data_root).expanduser().resolve()
        ev = load_raw_temporal_events(root.parent, root.name, config or {"data": {"format": "auto"}})
        src, dst, ts = ev.src.long(), ev.dst.long(), ev.ts
        eid = torch.arange(src.numel())
        if world_size > 1:
            mine = dst % world_size == rank
            src, dst, ts, eid = src[mine], dst[mine], ts[mine], eid[mine]
        return cls(src, dst, ts, ev.num_nodes, eid)

    # ------------------------------------------------------------------ temporal reads
    def neighbors_before(self, node: int, t: float) -> tuple[Tensor, Tensor, Tensor]:
        """(neighbours, timestamps, edge ids) of events into `node` strictly before `t`."""
        a, b = int(self.csr.rowptr[node]), int(self.csr.rowptr[node + 1])
        ts = self.csr.ts[a:b]
        end = a + int(torch.searchsorted(ts, torch.tensor(int(t)), side="left"))
        return self.csr.nbr[a:end], self.csr.ts[a:end], self.csr.eid[a:end]

    def slice_time(self, t0: float, t1: float) -> "TemporalGlobalCSR":
        m = (self.ts >= t0) & (self.ts < t1)
        return TemporalGlobalCSR(self.src[m], self.dst[m], self.ts[m], self._num_nodes, self.eid[m])
