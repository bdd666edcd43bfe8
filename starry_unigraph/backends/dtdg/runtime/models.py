"""Flare DTDG models (reference equations and parameter names:
backends/dtdg/runtime/models.py:102-248; the names are kept so checkpoints load
across the two frameworks).

* ``FlareEvolveGCN`` (EvolveGCN): the GCN weight evolves by a matrix GRU driven by
  a pooled graph context, W_t = MatGRU(W_{t-1}, pool_proj(mean(x))); the output
  head reads (A x) W_t.
* ``FlareTGCN`` (T-GCN, also ``gcn``): a two-layer GCN produces [u | r | c] of width
  3h; a reset-gated GRU cell updates h; the head reads h.
* ``FlareMPNNLSTM`` (MPNN-LSTM): a two-layer GCN of width h feeds two stacked LSTM
  cells whose four state tensors (h1, c1, h2, c2) travel with the window.

A model takes a window (``STGraphBlob``) or one graph. Over a window it walks
the window's steps; each step hands the carried state to its slot
(``step.fetch``: padded / mixed to the graph's rows) and back (``step.store``).
Every dense layer runs on the tcgen05 GEMM on CUDA (``starry_unigraph.ops.dtdg``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Callable

import torch
import torch.nn as nn

from starry_unigraph.ops.dtdg import linear, rgru_cell
from starry_unigraph.runtime.modules import GCNStack, MatGRUCell, _LSTMCell
from starry_unigraph.runtime.modules.gcn_layers import _gcn_message_pass, _graph_input

from .state import STGraphBlob, graph_steps


def _collect(blob_or_graph: Any, outputs: list[torch.Tensor]):
    """Per-step outputs for a window, the last output for a single graph."""
    return outputs if isinstance(blob_or_graph, STGraphBlob) else outputs[-1]


class FlareEvolveGCN(nn.Module):
    def __init__(self, input_size: int, hidden_size: int, output_size: int = 1) -> None:
        super().__init__()
        self.initial_weight = nn.Parameter(torch.empty(input_size, hidden_size))
        nn.init.xavier_uniform_(self.initial_weight)
        self.mat_gru = MatGRUCell(in_feats=input_size, out_feats=hidden_size)
        self.pool_proj = nn.Linear(input_size, input_size)
        self.out = nn.Linear(hidden_size, output_size)

    def _context(self, graph: Any) -> torch.Tensor:
        rows = _graph_input(graph).float()[: graph.num_dst_nodes]
        return linear(rows.mean(dim=0, keepdim=True), self.pool_proj.weight, self.pool_proj.bias)

    def forward(self, blob_or_graph: Any, state: torch.Tensor | None = None):
        w = state if state is not None else self.initial_weight
        preds = []
        for step in graph_steps(blob_or_graph):
            g = step.graph
            w = self.mat_gru(w, self._context(g))
            hidden = linear(_gcn_message_pass(g, _graph_input(g).float()), w.t().contiguous())
            preds.append(linear(hidden, self.out.weight, self.out.bias))
        return _collect(blob_or_graph, preds), w


class FlareTGCN(nn.Module):
    def __init__(self, input_size: int, hidden_size: int, output_size: int = 1) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.gcn = GCNStack(input_size, hidden_size * 3, num_layers=2)
        self.u_t = nn.Linear(hidden_size * 2, hidden_size)
        self.r_t = nn.Linear(hidden_size * 2, hidden_size)
        self.c_t = nn.Linear(hidden_size * 2, hidden_size)
        self.out = nn.Linear(hidden_size, output_size)

    def _cell(self, urc: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
        xu, xr, xc = urc.chunk(3, dim=-1)
        return rgru_cell(xu, xr, xc, h, self.u_t.weight, self.u_t.bias, self.r_t.weight, self.r_t.bias,
                         self.c_t.weight, self.c_t.bias)

    def forward(self, blob_or_graph: Any, state: torch.Tensor | None = None):
        steps = graph_steps(blob_or_graph)
        gates = self.gcn.layerwise(blob_or_graph)
        h = state
        preds = []
        for step, urc in zip(steps, gates):
            h = step.fetch(h)
            if h is None:
                h = urc.new_zeros(urc.size(0), self.hidden_size)
            h = self._cell(urc, h)
            step.store(h)
            preds.append(linear(h, self.out.weight, self.out.bias))
        return _collect(blob_or_graph, preds), h


class FlareMPNNLSTM(nn.Module):
    def __init__(self, input_size: int, hidden_size: int, output_size: int = 1) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.gcn = GCNStack(input_size, hidden_size, num_layers=2)
        self.rnn = nn.ModuleList([_LSTMCell(hidden_size, hidden_size), _LSTMCell(hidden_size, hidden_size)])
        self.out = nn.Linear(hidden_size, output_size)

    def _stack(self, x: torch.Tensor, carried: Any):
        """Both LSTM layers on one snapshot; `carried` is (h1, c1, h2, c2) or None."""
        states = []
        for layer, cell in enumerate(self.rnn):
            prev = None if carried is None else tuple(carried[2 * layer: 2 * layer + 2])
            x, c = cell(x, prev)
            states.extend((x, c))
        return x, tuple(states)

    def forward(self, blob_or_graph: Any, state: Any = None):
        steps = graph_steps(blob_or_graph)
        feats = self.gcn.layerwise(blob_or_graph)
        carried = state
        preds = []
        for step, x in zip(steps, feats):
            top, carried = self._stack(x, step.fetch(carried))
            step.store(carried)
            preds.append(linear(top, self.out.weight, self.out.bias))
        return _collect(blob_or_graph, preds), carried


@dataclass(frozen=True)
class FlareModelSpec:
    model_cls: type[nn.Module]


# registry names of the reference (``gcn`` runs T-GCN)
MODEL_SPECS: dict[str, FlareModelSpec] = {name: FlareModelSpec(cls) for name, cls in (
    ("evolvegcn", FlareEvolveGCN), ("tgcn", FlareTGCN), ("mpnn_lstm", FlareMPNNLSTM), ("gcn", FlareTGCN))}


def build_flare_model(model_name: str, input_size: int, hidden_size: int, output_size: int) -> nn.Module:
    spec = MODEL_SPECS.get(model_name.lower())
    if spec is None:
        raise KeyError(f"Unsupported flare model: {model_name} (known: {sorted(MODEL_SPECS)})")
    return spec.model_cls(input_size=input_size, hidden_size=hidden_size, output_size=output_size)


def extract_graph_labels(blob_or_graph: Any) -> torch.Tensor | None:
    steps = graph_steps(blob_or_graph)
    if not steps:
        return None
    g = steps[-1].graph
    y = g.dstdata.get("y")
    if y is None and "y" in g.srcdata:
        y = g.srcdata["y"][: g.num_dst_nodes]
    if y is None:
        return None
    return y.view(-1, 1) if y.dim() == 1 else y
