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
    def __init__(self, ctdg_session: Any, max_batch: int | None = None):
        """`max_batch`: cap on the events per unit (the CUDA step holds one configured batch)."""
        self.session = ctdg_session
        self.max_batch = max_batch
        self._csr_cpu: dict[str, Any] = {}  # host copy of each split's T-CSR, made once

    def iter_batches(self, split: str, batch_size: int) -> Iterator[ChunkAtomic]:
        rt = self.session.online_runtime
        if self.max_batch is not None and rt.engine is not None:
            batch_size = min(int(batch_size), int(self.max_batch))
        split = "test" if split == "predict" else split
        if split not in self._csr_cpu:
            csr = rt.sampler.csr(split)
            self._csr_cpu[split] = type(csr)(csr.rowptr.cpu(), csr.nbr.cpu(), csr.eid.cpu(), csr.ts.cpu(),
                                             csr.num_nodes)
        csr_cpu = self._csr_cpu[split]
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
        """The loader's steps in lock-step order: each a chunk restricted to the step's
        events (its T-CSR kept), or an empty unit for a padding step."""
        from dataclasses import replace

        split = "test" if split == "predict" else split
        for unit in self.loader._splits[split]:
            if unit is None:
                z = torch.zeros(0, dtype=torch.long)
                yield _events_chunk(-1, z, z, torch.zeros(0), z)
                continue
            chunk, lo, hi = unit
            ev = chunk.events
            yield replace(chunk, events={k: ev[k][lo:hi] for k in ("src", "dst", "ts", "eid")})

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


class RuntimeStepModel:
    """The session's runtime as the unified engine's ``TemporalModel``.

    ``predict(state, batch)`` runs the mode's own step on the unit the batch was
    materialised from (``batch.source``): the CTDG step on the unit's events (the
    fused sm_100a step on CUDA; chunk mode steps are CTDG steps too), or the Flare
    window step of a DTDG unit. In train mode it is a training step (forward,
    backward, optimizer). It returns the step result, whose loss is a float and whose
    metrics sit under ``meta``: the task adapters read both from it, and the engine
    takes no second backward or optimizer step.
    """

    def __init__(self, session: Any):
        self.session = session
        self.training = True
        self.current_split = "train"

    def train(self, mode: bool = True) -> "RuntimeStepModel":
        """Set at the start of every engine epoch. An evaluation epoch of a DTDG session
        starts from a fresh recurrent state, as the session's own evaluation does."""
        self.training = bool(mode)
        runtime = getattr(self.session, "runtime", None)
        if not mode and self.session.ctdg_session is None and runtime is not None:
            runtime.state.pop("eval_rnn_state", None)
        return self

    def eval(self) -> "RuntimeStepModel":
        return self.train(False)

    def _ctdg_runtime(self):
        s = self.session
        if s.ctdg_session is not None:
            return s.ctdg_session.online_runtime
        return getattr(s.snapshot_core, "_ctdg", None)

    def predict(self, state: Any, batch: Any) -> dict[str, Any]:
        from starry_unigraph.backends.ctdg.runtime.data import CTDGDataBatch

        unit = batch.source
        split = "test" if self.current_split == "predict" else self.current_split
        ev = unit.events
        if "item" in ev:  # a Flare window
            loader, runtime = self.session.snapshot_core, self.session.runtime
            return loader.run_train_step(runtime, ev["item"]) if self.training else \
                loader.run_eval_step(runtime, ev["item"])
        rt = self._ctdg_runtime()
        b = CTDGDataBatch(index=unit.chunk_id[0], split=split, event_ids=ev["eid"], src=ev["src"], dst=ev["dst"],
                          ts=ev["ts"], edge_feat=rt.dataset.edge_feat[ev["eid"]])
        return rt.train_step(b) if self.training else rt.eval_step(b, split)
