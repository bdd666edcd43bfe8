"""RNN state management over a sliding window of snapshots
(reference backends/dtdg/runtime/state.py:22-346).

``RNNStateManager`` keeps the window's graphs and patches each with
``flare_fetch_state`` / ``flare_store_state``:
  * ``pad``: state rows are zero-padded / truncated to the graph's node count
    (and forgotten between steps),
  * ``mix``: missing rows are filled from the detached state stored for that
    window slot in the previous step.
Older window slots may be truncated to the first ``end`` nodes of the
chunk-permuted order (temporal decay); truncated graphs drop their halo.
"""
from __future__ import annotations

import types
from typing import Any

import torch
import torch.nn.functional as F
from torch import Tensor

from starry_unigraph.data.partition import SnapshotBlock


class RNNStateManager:
    def __init__(self, ends_list: list[int | None], mode: str = "pad", disable_routes: bool = False) -> None:
        ends_list = [e for e in ends_list if e is None or e > 0]
        self._ends_list = ends_list
        self._state_list: list[Any] = [None] * len(ends_list)
        self._graph_list: list[Any] = []
        self._mode = mode
        self._disable_routes = disable_routes
        self._snapshot_count = 0

    def __len__(self) -> int:
        return len(self._graph_list)

    def __getitem__(self, i: int) -> Any:
        return self._graph_list[i]

    @classmethod
    def patch_dummy_methods(cls, g: Any) -> Any:
        g.flare_snapshot_id = getattr(g, "flare_snapshot_id", -1)
        g.flare_rnn_state_idx = -1
        g.flare_is_full_snapshot = True
        g.flare_fetch_state = types.MethodType(lambda self, x, end=None: x, g)
        g.flare_store_state = types.MethodType(lambda self, x: None, g)
        return g

    def add(self, g: Any) -> None:
        while len(self._graph_list) >= len(self._state_list):
            self._graph_list.pop(0)
        self._graph_list = [self._patch(h) for h in self._graph_list]
        self._graph_list.append(self._patch(g))

    def _patch(self, g: Any) -> Any:
        snap = getattr(g, "flare_snapshot_id", None)
        if snap is None:
            snap = self._snapshot_count
            self._snapshot_count += 1
        idx = getattr(g, "flare_rnn_state_idx", len(self._ends_list)) - 1
        end = self._ends_list[idx]
        if self._disable_routes or end is not None:
            base = getattr(g, "_untruncated", g)
            g = self._truncate_graph(base, end)
            g._untruncated = base
        g.flare_rnn_state_idx = idx
        g.flare_fetch_state = types.MethodType(self._fetch, g)
        g.flare_store_state = types.MethodType(self._store, g)
        g.flare_snapshot_id = snap
        g.flare_is_full_snapshot = end is None
        return g

    def _fetch(self, this: Any, state: Any, end: int | None = None) -> Any:
        old = self._state_list[this.flare_rnn_state_idx]
        if end is None:
            end = this.num_dst_nodes
        if old is None or self._mode == "pad":
            return self.state_padding(state, end)
        if self._mode == "mix":
            return self.state_mixing(state, old, end)
        raise ValueError(f"Unknown mode: {self._mode}")

    def _store(self, this: Any, state: Any) -> None:
        if self._mode == "pad":
            self._state_list[this.flare_rnn_state_idx] = None
        elif self._mode == "mix":
            self._state_list[this.flare_rnn_state_idx] = self.state_detach(state)
        else:
            raise ValueError(f"Unknown mode: {self._mode}")

    @classmethod
    def apply_state(cls, fn, state: Any, old_state: Any = None) -> Any:
        if isinstance(state, (tuple, list)):
            olds = old_state if old_state is not None else [None] * len(state)
            res = [fn(s, t) if old_state is not None else fn(s) for s, t in zip(state, olds)]
            return tuple(res) if isinstance(state, tuple) else res
        if isinstance(state, dict):
            return {k: (fn(v, old_state[k]) if old_state is not None else fn(v)) for k, v in state.items()}
        return fn(state) if old_state is None else fn(state, old_state)

    @classmethod
    def state_detach(cls, state: Any) -> Any:
        return cls.apply_state(lambda s: s.detach() if isinstance(s, Tensor) else s, state)

    @classmethod
    def state_padding(cls, state: Any, end: int) -> Any:
        def pad(s):
            if not isinstance(s, Tensor):
                return s
            n = s.size(0)
            if n > end:
                return s[:end]
            if n < end:
                return F.pad(s, [0] * (s.dim() * 2 - 1) + [end - n])
            return s

        return cls.apply_state(pad, state)

    @classmethod
    def state_mixing(cls, state: Any, old_state: Any, end: int) -> Any:
        def mix(cur, old):
            if not isinstance(cur, Tensor):
                return cur
            if cur.size(0) >= end:
                return cur[:end]
            need = end - cur.size(0)
            tail = old[cur.size(0):end] if old.size(0) >= end else \
                F.pad(old[cur.size(0):], [0] * (old.dim() * 2 - 1) + [end - old.size(0)])
            return torch.cat([cur, tail[:need]], dim=0)

        return cls.apply_state(mix, state, old_state)

    @classmethod
    def _truncate_graph(cls, g: SnapshotBlock, end: int | None) -> SnapshotBlock:
        n_dst = g.num_dst_nodes
        end = n_dst if end is None else min(end, n_dst)
        keep = (g.edge_src < end) & (g.edge_dst < end)
        out = SnapshotBlock(num_src_nodes=end, num_dst_nodes=end, edge_src=g.edge_src[keep], edge_dst=g.edge_dst[keep])
        for k, v in g.srcdata.items():
            out.dstdata[k] = v[:end]
        for k, v in g.dstdata.items():
            out.dstdata[k] = v[:end]
        for k, v in g.edata.items():
            out.edata[k] = v[keep]
        out.route = None
        out.is_block = False
        out.graph_meta = dict(g.graph_meta)
        return out


class STWindowState:
    def __init__(self, full_snapshot_limit: int = 1) -> None:
        self.full_snapshot_limit = full_snapshot_limit

    def describe(self) -> dict[str, Any]:
        return {"full_snapshot_limit": self.full_snapshot_limit}


class STGraphBlob:
    def __init__(self, state: RNNStateManager) -> None:
        self.state = state

    def __len__(self) -> int:
        return len(self.state)

    def __getitem__(self, idx: int) -> Any:
        return self.state[idx]

    def __iter__(self):
        for i in range(len(self)):
            yield self.state[i]

    @property
    def current_graph(self) -> Any:
        return self.state[-1]

    @property
    def flare_is_full_snapshot(self) -> bool:
        return bool(getattr(self.current_graph, "flare_is_full_snapshot", True))

    @property
    def snapshot_index(self) -> int:
        return int(getattr(self.current_graph, "flare_snapshot_id", 0))

    def describe(self) -> dict[str, Any]:
        return {"len": len(self), "snapshot_index": self.snapshot_index, "is_full_snapshot": self.flare_is_full_snapshot}
