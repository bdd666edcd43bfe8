"""Adapters exposing the CTDG runtime, the Flare loader and the chunk loader as
``GraphBackend``s of the unified pipeline (reference runtime/backend_adapters.py:20-194,
where the chunks were empty placeholders; here they carry the batch's events and
temporal neighbourhood)."""
from __future__ import annotations

from typing import Any, Iterator

import torch
from torch import Tensor

from starry_unigraph.data.chunk_atomic import ChunkAtomic

from .backend import GraphBackend, StateManager


def _events_chunk(idx: int, src: Tensor, dst: Tensor, ts: Tensor, eid: Tensor, csr=None) -> ChunkAtomic:
    nodes = torch.unique(torch.cat([src, dst])) if src.numel() else torch.zeros(0, dtype=torch.long)
    if csr is not None and nodes.numel():
        lo, hi = csr.rowptr[nodes], csr.rowptr[nodes + 1]
        seg = [torch.arange(int(a), int(b)) for a, b in zip(lo.tolist(), hi.tolist())]
        sel = torch.cat(seg) if seg else torch.zeros(0, dtype=torch.long)
        rowptr = torch.zeros(nodes.numel() + 1, dtype=torch.long)
        rowptr[1:] = torch.cumsum(hi - lo, 0)
        col, tts, eids = csr.nbr[sel], csr.ts[sel], csr.eid[sel]
    else:
        rowptr = torch.zeros(nodes.numel() + 1, dtype=torch.long)
        col = tts = eids = torch.zeros(0, dtype=torch.long)
    z = torch.zeros(0, dtype=torch.long)
    tr = (float(ts.min()), float(ts.max())) if ts.numel() else (0.0, 0.0)
    return ChunkAtomic(chunk_id=(idx, 0), time_range=tr, node_set=nodes, tcsr_rowptr=rowptr, tcsr_col=col.cpu(),
                       tcsr_ts=tts.cpu(), tcsr_edge_id=eids.cpu(), cross_node_ids=z, cross_node_home=z,
                       cross_edge_count=z, load_estimate=float(src.numel()),
                       events={"src": src, "dst": dst, "ts": ts, "eid": eid})


class CTDGGraphBackend(GraphBackend):
    def __init__(self, ctdg_session: Any):
        self.session = ctdg_session

    def iter_batches(self, split: str, batch_size: int) -> Iterator[ChunkAtomic]:
        rt = self.session.online_runtime
        csr = rt.sampler.csr("test" if split == "predict" else split)
        csr_cpu = type(csr)(csr.rowptr.cpu(), csr.nbr.cpu(), csr.eid.cpu(), csr.ts.cpu(), csr.num_nodes)
        for b in rt.iter_batches(split, batch_size):
            yield _events_chunk(b.index, b.src, b.dst, b.ts, b.event_ids, csr_cpu)

    def reset(self) -> None:
        return None

    def describe(self) -> dict[str, Any]:
        return {"backend": "ctdg_online", **self.session.online_runtime.dataset.describe()}


class FlareGraphBackend(GraphBackend):
    def __init__(self, flare_loader: Any):
        self.loader = flare_loader

    def iter_batches(self, split: str, batch_size: int) -> Iterator[ChunkAtomic]:
        it = self.loader.iter_train() if split == "train" else self.loader.iter_eval(split)
        for i, item in enumerate(it):
            g = item.current_graph if hasattr(item, "current_graph") else item.graph
            src_ids = g.srcdata.get("_ID", torch.arange(g.num_src_nodes))
            s, d = src_ids[g.edge_src.long()].cpu(), g.dstdata.get("_ID", torch.arange(g.num_dst_nodes))[
                g.edge_dst.long()].cpu()
            ch = _events_chunk(i, s, d, torch.full((s.numel(),), float(i)), torch.arange(s.numel()))
            ch.events["graph"] = g
            ch.events["item"] = item
            yield ch

    def reset(self) -> None:
        return None

    def describe(self) -> dict[str, Any]:
        return {"backend": "flare", **self.loader.build_snapshot_index()}


class ChunkGraphBackend(GraphBackend):
    def __init__(self, chunk_loader: Any):
        self.loader = chunk_loader

    def iter_batches(self, split: str, batch_size: int) -> Iterator[ChunkAtomic]:
        yield from self.loader.iter_chunks(split)

    def reset(self) -> None:
        return None

    def describe(self) -> dict[str, Any]:
        return {"backend": "chunk", **self.loader.chunk_manifest}


class DummyStateManager(StateManager):
    """Stateless manager (models that carry no recurrent state between batches)."""

    def __init__(self):
        self.calls = 0

    def prepare(self, node_ids: Tensor, timestamps: Tensor | None = None) -> dict[str, Any]:
        self.calls += 1
        return {}

    def update(self, model_output: dict[str, Tensor], chunk: ChunkAtomic) -> None:
        return None

    def reset(self) -> None:
        self.calls = 0

    def describe(self) -> dict[str, Any]:
        return {"manager": "dummy", "calls": self.calls}
