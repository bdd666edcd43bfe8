"""Sliding training windows of snapshot graphs and the RNN state carried between
them (reference behaviour: backends/dtdg/runtime/state.py:22-346).

A window has ``len(ends_list)`` slots, the newest snapshot in the last slot.
Slot ``s`` may truncate its graph to the first ``ends_list[s]`` nodes of the
chunk-permuted order (temporal decay; ``None`` keeps the whole graph, and a
truncated graph drops its halo). Every slot also owns a state cell:

* ``pad``: a slot's incoming state is zero-padded or cut to the graph's rows and
  nothing is remembered between windows;
* ``mix``: rows missing from the incoming state are taken from the detached
  state this slot produced in the previous window.

Design: the slot states live in ``RNNStateManager`` (owned by the loader that
slides the window); graphs are never modified. ``add`` returns nothing, and
``snapshot()`` freezes the current window into an ``STGraphBlob`` whose steps
carry explicit ``fetch`` / ``store`` closures bound to their slot, so a blob kept
for later (a pre-built list of windows, a captured CUDA graph) still describes
its own window after the loader has moved on.
"""
from __future__ import annotations

from collections import deque
from dataclasses import dataclass, field
from typing import Any, Callable

import torch
import torch.nn.functional as F
from torch import Tensor

from starry_unigraph.data.partition import SnapshotBlock


# ---------------------------------------------------------------------------
# state transforms (tensor, tuple / list or dict of tensors)
# ---------------------------------------------------------------------------
def _map_state(fn: Callable[..., Any], state: Any, other: Any = None) -> Any:
    if isinstance(state, dict):
        return {k: _map_state(fn, v, None if other is None else other[k]) for k, v in state.items()}
    if isinstance(state, (tuple, list)):
        parts = [_map_state(fn, s, None if other is None else other[i]) for i, s in enumerate(state)]
        return tuple(parts) if isinstance(state, tuple) else parts
    if not isinstance(state, Tensor):
        return state
    return fn(state) if other is None else fn(state, other)


def _fit_rows(t: Tensor, rows: int) -> Tensor:
    """First `rows` rows of `t`, zero rows appended when it is shorter."""
    if t.size(0) >= rows:
        return t[:rows]
    return F.pad(t, [0, 0] * (t.dim() - 1) + [0, rows - t.size(0)])


def _complete_rows(cur: Tensor, old: Tensor, rows: int) -> Tensor:
    """`cur` extended to `rows` rows with the rows of `old` that follow it."""
    if cur.size(0) >= rows:
        return cur[:rows]
    tail = _fit_rows(old[cur.size(0):], rows - cur.size(0))
    return torch.cat([cur, tail], dim=0)


@dataclass
class WindowStep:
    """One snapshot of a frozen window: its (possibly truncated) graph and the
    state hooks of the slot it occupies."""

    graph: Any
    slot: int
    snapshot_id: int
    full: bool
    fetch: Callable[[Any], Any]
    store: Callable[[Any], None]


def _identity(state: Any) -> Any:
    return state


def _discard(state: Any) -> None:
    return None


def graph_steps(blob_or_graph: Any) -> list[WindowStep]:
    """The steps of a window, or one stateless step for a bare graph."""
    if isinstance(blob_or_graph, STGraphBlob):
        return list(blob_or_graph.steps)
    g = blob_or_graph
    return [WindowStep(g, -1, int(getattr(g, "flare_snapshot_id", -1)), True, _identity, _discard)]


class RNNStateManager:
    """Window slots (truncation + carried state) of one training pass."""

    def __init__(self, ends_list: list[int | None], mode: str = "pad", disable_routes: bool = False) -> None:
        if mode not in ("pad", "mix"):
            raise ValueError(f"Unknown mode: {mode}")
        self.ends: list[int | None] = [e for e in ends_list if e is None or e > 0] or [None]
        self.mode = mode
        self.disable_routes = bool(disable_routes)
        self.cells: list[Any] = [None] * len(self.ends)   # carried state per slot (mix mode)
        self._graphs: deque = deque(maxlen=len(self.ends))
        self._views: dict[tuple[int, int | None], Any] = {}  # (id(graph), end) -> truncated view
        self._next_id = 0

    @property
    def _mode(self) -> str:  # name the step-graph capture checks
        return self.mode

    @property
    def capacity(self) -> int:
        return len(self.ends)

    def add(self, graph: Any) -> None:
        """Slide the window by one snapshot (the oldest leaves when the window is full)."""
        if getattr(graph, "flare_snapshot_id", None) is None:
            graph.flare_snapshot_id = self._next_id
        self._next_id += 1
        if len(self._graphs) == self._graphs.maxlen:
            gone = self._graphs[0]
            for key in [k for k in self._views if k[0] == id(gone)]:
                del self._views[key]
        self._graphs.append(graph)

    def slot_of(self, position: int) -> int:
        """Slot of the window's `position`-th graph (0 = oldest present)."""
        return self.capacity - len(self._graphs) + position

    def _view(self, graph: Any, end: int | None) -> Any:
        if end is None and not self.disable_routes:
            return graph
        key = (id(graph), end)
        if key not in self._views:
            self._views[key] = truncate_block(graph, end)
        return self._views[key]

    def fetch(self, slot: int, state: Any, rows: int) -> Any:
        old = self.cells[slot]
        if state is None and old is None:
            return None
        if self.mode == "pad" or old is None:
            return _map_state(lambda t: _fit_rows(t, rows), state)
        return _map_state(lambda cur, prev: _complete_rows(cur, prev, rows), state, old)

    def store(self, slot: int, state: Any) -> None:
        self.cells[slot] = _map_state(lambda t: t.detach(), state) if self.mode == "mix" else None

    def snapshot(self) -> "STGraphBlob":
        steps = []
        for pos, graph in enumerate(self._graphs):
            slot = self.slot_of(pos)
            end = self.ends[slot]
            view = self._view(graph, end)
            rows = int(view.num_dst_nodes)
            steps.append(WindowStep(
                graph=view, slot=slot, snapshot_id=int(graph.flare_snapshot_id), full=end is None,
                fetch=lambda state, s=slot, n=rows: self.fetch(s, state, n),
                store=lambda state, s=slot: self.store(s, state)))
        return STGraphBlob(self, steps)

    # helpers kept under the reference's names for callers of the old static API
    @staticmethod
    def state_detach(state: Any) -> Any:
        return _map_state(lambda t: t.detach(), state)

    @staticmethod
    def state_padding(state: Any, end: int) -> Any:
        return _map_state(lambda t: _fit_rows(t, end), state)

    @staticmethod
    def state_mixing(state: Any, old_state: Any, end: int) -> Any:
        return _map_state(lambda cur, prev: _complete_rows(cur, prev, end), state, old_state)

    def __len__(self) -> int:
        return len(self._graphs)

    def __getitem__(self, i: int) -> Any:
        return self.snapshot().steps[i].graph


def truncate_block(g: SnapshotBlock, end: int | None) -> SnapshotBlock:
    """The block restricted to its first `end` destination nodes (and the edges
    among them), without halo rows or route."""
    keep_n = g.num_dst_nodes if end is None else min(int(end), g.num_dst_nodes)
    edge_mask = (g.edge_src < keep_n) & (g.edge_dst < keep_n)
    out = SnapshotBlock(num_src_nodes=keep_n, num_dst_nodes=keep_n, edge_src=g.edge_src[edge_mask],
                        edge_dst=g.edge_dst[edge_mask])
    for table in (g.srcdata, g.dstdata):
        for name, value in table.items():
            out.dstdata[name] = value[:keep_n]
    out.edata.update({name: value[edge_mask] for name, value in g.edata.items()})
    out.route = None
    out.is_block = False
    out.graph_meta = dict(g.graph_meta)
    out.flare_snapshot_id = getattr(g, "flare_snapshot_id", -1)
    return out


@dataclass
class STWindowState:
    full_snapshot_limit: int = 1

    def describe(self) -> dict[str, Any]:
        return {"full_snapshot_limit": self.full_snapshot_limit}


@dataclass
class STGraphBlob:
    """A frozen window: its steps (graphs + slot hooks) in time order."""

    state: RNNStateManager
    steps: list[WindowStep] = field(default_factory=list)

    def __len__(self) -> int:
        return len(self.steps)

    def __getitem__(self, idx: int) -> Any:
        return self.steps[idx].graph

    def __iter__(self):
        return (s.graph for s in self.steps)

    @property
    def current_graph(self) -> Any:
        return self.steps[-1].graph

    @property
    def flare_is_full_snapshot(self) -> bool:
        return self.steps[-1].full if self.steps else True

    @property
    def snapshot_index(self) -> int:
        return self.steps[-1].snapshot_id if self.steps else 0

    def describe(self) -> dict[str, Any]:
        return {"len": len(self), "snapshot_index": self.snapshot_index, "is_full_snapshot": self.flare_is_full_snapshot}
