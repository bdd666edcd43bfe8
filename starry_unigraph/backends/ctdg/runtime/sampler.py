"""Temporal neighbour sampling over a T-CSR keyed by destination.

Semantics of the reference BTS sampler (vendor/bts_sampler/sampler/include/sampler.h:213-399,
neighbors.h:243-267): a root's candidates are the sources of events *into* it,
kept in stream (time) order; ``end = lower_bound(ts, root_ts)`` keeps strictly
earlier events; ``recent`` takes the last min(k, end) candidates, ``uniform``
draws k with replacement when more than k are available (all of them
otherwise). Timestamps are truncated to int64 as the reference does.

``TemporalCSR`` is built once per split (stable sort by destination preserves
time order inside each list). On CUDA the arrays live on the device and the
sampler is the sm_100a warp-per-root kernel; the host C++ sampler
(``starry_unigraph._native``) and the vectorised torch fallback serve CPU runs
and act as the oracle.

``recent`` and ``uniform`` run vectorised over the T-CSR (and in the CUDA step).
The other policies of the native sampler, ``weighted`` (draws proportional to
the events' weights), ``boundery_recent_uniform`` and ``boundery_recent_decay``
(remote candidates, whose event or neighbour another rank owns, kept with a
probability), run in the host sampler on CPU and come back in the same dense
[roots, k] block layout; the CUDA step does not implement them.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .data import TGTemporalDataset
from .models import DenseBlock

_KEY_SHIFT = 40  # (node << 40) | ts keeps (dst, ts) order in one int64 key


@dataclass
class TemporalCSR:
    rowptr: torch.Tensor  # [N + 1] int64
    nbr: torch.Tensor     # [E] int64 (source of the event)
    eid: torch.Tensor     # [E] int64
    ts: torch.Tensor      # [E] int64 (truncated)
    num_nodes: int
    _keys: torch.Tensor | None = None  # (node << 40) | ts per entry, built on first use

    def keys(self) -> torch.Tensor:
        """Sorted (node, ts) search keys of every entry, computed once per T-CSR."""
        if self._keys is None:
            node_of = torch.repeat_interleave(torch.arange(self.num_nodes, device=self.rowptr.device),
                                              self.rowptr[1:] - self.rowptr[:-1])
            self._keys = (node_of << _KEY_SHIFT) | self.ts
        return self._keys

    @classmethod
    def build(cls, row: torch.Tensor, col: torch.Tensor, eid: torch.Tensor, ts: torch.Tensor, num_nodes: int,
              device: str | torch.device = "cpu") -> "TemporalCSR":
        dev = torch.device(device)
        row, col, eid, ts = (t.to(dev) for t in (row.long(), col.long(), eid.long(), ts.long()))
        order = torch.argsort(col, stable=True)
        counts = torch.bincount(col, minlength=num_nodes)
        rowptr = torch.zeros(num_nodes + 1, dtype=torch.long, device=dev)
        rowptr[1:] = torch.cumsum(counts, 0)
        return cls(rowptr=rowptr, nbr=row[order].contiguous(), eid=eid[order].contiguous(),
                   ts=ts[order].contiguous(), num_nodes=num_nodes)

    def sample_torch(self, roots: torch.Tensor, root_ts: torch.Tensor, k: int, policy: str = "recent",
                     generator: torch.Generator | None = None) -> DenseBlock:
        """Vectorised reference implementation (CPU oracle)."""
        dev = self.rowptr.device
        roots = roots.to(dev).long()
        rts = root_ts.to(dev).long()
        lo = self.rowptr[roots]
        hi = self.rowptr[roots + 1]
        end = torch.searchsorted(self.keys(), (roots << _KEY_SHIFT) | rts, side="left")
        end = torch.minimum(torch.maximum(end, lo), hi)
        avail = end - lo
        j = torch.arange(k, device=dev).unsqueeze(0)
        if policy == "recent":
            cnt = torch.clamp(avail, max=k)
            pos = end.unsqueeze(1) - cnt.unsqueeze(1) + j
        else:
            cnt = torch.where(avail <= k, avail, torch.full_like(avail, k))
            rnd = torch.randint(0, 2**62, (roots.numel(), k), generator=generator).to(dev)
            draw = lo.unsqueeze(1) + rnd % avail.clamp(min=1).unsqueeze(1)
            take_all = end.unsqueeze(1) - cnt.unsqueeze(1) + j
            pos = torch.where((avail <= k).unsqueeze(1), take_all, draw)
        valid = j < cnt.unsqueeze(1)
        if self.nbr.numel() == 0:  # no events at all: every slot is empty
            none = torch.full(pos.shape, -1, dtype=torch.long, device=dev)
            return DenseBlock(roots=roots, nbr=none, eid=none.clone(), dt=torch.zeros(pos.shape, device=dev),
                              count=torch.zeros_like(cnt, dtype=torch.int32))
        pos = torch.where(valid, pos, torch.zeros_like(pos))
        nbr = torch.where(valid, self.nbr[pos], torch.full_like(pos, -1))
        eid = torch.where(valid, self.eid[pos], torch.full_like(pos, -1))
        dt = torch.where(valid, (rts.unsqueeze(1) - self.ts[pos]).float(), torch.zeros(pos.shape, device=dev))
        return DenseBlock(roots=roots, nbr=nbr, eid=eid, dt=dt, count=cnt.int())


@dataclass
class CTDGSampleOutput:
    split: str
    root_nodes: torch.Tensor
    timestamps: torch.Tensor
    blocks: list[DenseBlock]

    @property
    def sampled_nodes(self) -> torch.Tensor:
        """Roots and every sampled neighbour, unique (computed once: read by the remote
        pull and by the step's description)."""
        cached = self.__dict__.get("_sampled_nodes")
        if cached is None:
            parts = [self.root_nodes] + [b.nbr[b.mask()] for b in self.blocks]
            cached = self.__dict__["_sampled_nodes"] = torch.unique(torch.cat(parts))
        return cached

    @property
    def sampled_eids(self) -> torch.Tensor:
        if not self.blocks:
            return torch.empty(0, dtype=torch.long)
        return torch.unique(torch.cat([b.eid[b.mask()] for b in self.blocks]))

    def describe(self) -> dict[str, int]:
        return {"root_count": int(self.root_nodes.numel()), "sampled_node_count": int(self.sampled_nodes.numel()),
                "sampled_edge_count": int(self.sampled_eids.numel()), "num_layers": len(self.blocks)}


class NativeTemporalSampler:
    """Multi-hop temporal sampler over per-split T-CSRs (built lazily, cached).

    Layer i+1 roots are layer i's sampled neighbours with their event times
    (reference sampler.h:393-399).
    """

    def __init__(self, dataset: TGTemporalDataset, fanout: list[int], history: int, strategy: str,
                 workers: int = 1, device: str | torch.device = "cpu", boundary_p: float = 1.0):
        from starry_unigraph.native.bts_sampler import SAMPLER_POLICIES

        if strategy not in SAMPLER_POLICIES:
            raise ValueError(f"unknown sampling strategy {strategy!r} (one of {SAMPLER_POLICIES})")
        self.dataset = dataset
        self.fanout = list(fanout)
        self.history = int(history)
        self.strategy = str(strategy)
        self.workers = int(workers)
        self.device = torch.device(device)
        self.boundary_p = float(boundary_p)
        self._csr: dict[str, TemporalCSR] = {}
        self._native: dict[str, object] = {}

    def csr(self, split: str) -> TemporalCSR:
        split = "test" if split == "predict" else split
        if split not in self._csr:
            g = self.dataset.sampler_graph(split)
            self._csr[split] = TemporalCSR.build(g["row"], g["col"], g["eid"], g["ts"], self.dataset.num_nodes,
                                                 self.device)
        return self._csr[split]

    def _native_sampler(self, split: str):
        from starry_unigraph.native.bts_sampler import BTSNativeSampler, build_temporal_neighbor_block

        split = "test" if split == "predict" else split
        if split not in self._native:
            g = self.dataset.sampler_graph(split)
            tnb = build_temporal_neighbor_block(f"su_{id(self)}_{split}", g["row"], g["col"], self.dataset.num_nodes,
                                                g["eid"], edge_weight=g["weight"], timestamp=g["ts"])
            ds = self.dataset
            parts = getattr(ds, "node_parts", None)
            kw = {}
            if parts is not None and self.strategy.startswith("boundery"):
                kw = {"local_part": int(ds.partition_rank), "node_part": parts,
                      "edge_part": ds.edge_parts if ds.edge_parts is not None else parts[ds.src]}
            self._native[split] = BTSNativeSampler(tnb, ds.num_nodes, ds.num_edges, self.history, self.fanout,
                                                   workers=self.workers, policy=self.strategy,
                                                   probability=self.boundary_p, **kw)
        return self._native[split]

    def _sample_native(self, split: str, root_nodes: torch.Tensor, timestamps: torch.Tensor) -> CTDGSampleOutput:
        """Host sampler, its flat per-layer output laid out as [roots, k] blocks (k = the
        layer's fanout, or more where a boundary policy kept more)."""
        blocks_out = self._native_sampler(split).sample_from_nodes(root_nodes.long().cpu(), timestamps.long().cpu())
        roots = root_nodes.long().cpu()
        blocks: list[DenseBlock] = []
        for layer, b in enumerate(blocks_out):
            k = self.fanout[min(layer, len(self.fanout) - 1)]
            src = b.src_index()
            count = torch.bincount(src, minlength=roots.numel()) if src.numel() else \
                torch.zeros(roots.numel(), dtype=torch.long)
            width = max(k, int(count.max()) if count.numel() else 0)
            first = torch.cumsum(count, 0) - count
            col = torch.arange(src.numel()) - first[src] if src.numel() else src
            nbr = torch.full((roots.numel(), width), -1, dtype=torch.long)
            eid = nbr.clone()
            dt = torch.zeros(roots.numel(), width)
            nbr[src, col] = b.sample_nodes()
            eid[src, col] = b.eid()
            dt[src, col] = b.delta_ts().float()
            blocks.append(DenseBlock(roots=roots, nbr=nbr.to(self.device), eid=eid.to(self.device),
                                     dt=dt.to(self.device), count=count.int().to(self.device)))
            roots = b.sample_nodes()
        return CTDGSampleOutput(split=split, root_nodes=root_nodes.long(), timestamps=timestamps.float(), blocks=blocks)

    def sample(self, split: str, root_nodes: torch.Tensor, timestamps: torch.Tensor) -> CTDGSampleOutput:
        if self.strategy not in ("recent", "uniform"):
            return self._sample_native(split, root_nodes, timestamps)
        csr = self.csr(split)
        blocks: list[DenseBlock] = []
        roots, rts = root_nodes.long(), timestamps.long()
        for layer in range(max(1, self.history)):
            k = self.fanout[min(layer, len(self.fanout) - 1)]
            blk = csr.sample_torch(roots, rts, k, self.strategy)
            blocks.append(blk)
            m = blk.mask()
            roots = blk.nbr[m]
            rts = (rts.to(blk.dt.device).unsqueeze(1) - blk.dt.long())[m]
        return CTDGSampleOutput(split=split, root_nodes=root_nodes.long(), timestamps=timestamps.float(), blocks=blocks)
