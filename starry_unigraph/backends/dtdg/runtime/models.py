"""Flare DTDG models (reference backends/dtdg/runtime/models.py:31-295).

* ``FlareEvolveGCN`` (EvolveGCN): W_t = MatGRU(W_{t-1}, pool_proj(mean(x))),
  out = Linear((A x) W_t).
* ``FlareTGCN`` (T-GCN; also serves ``gcn``): urc = GCNStack(F -> 3h), GRU-style
  gates u, r, c, h' = u h + (1 - u) c, out = Linear(h).
* ``FlareMPNNLSTM`` (MPNN-LSTM): GCNStack(F -> h, 2 layers) then two stacked
  LSTM cells, state (h1, c1, h2, c2) carried through the window's state manager.
Every dense layer runs on the tcgen05 GEMM on CUDA (``starry_unigraph.ops.dtdg``).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.nn as nn

from starry_unigraph.ops.dtdg import linear, rgru_cell
from starry_unigraph.runtime.modules import GCNStack, MatGRUCell, _LSTMCell
from starry_unigraph.runtime.modules.gcn_layers import _gcn_message_pass, _graph_input

from .state import STGraphBlob


def _graph_sequence(blob_or_graph) -> list[Any]:
    return list(blob_or_graph) if isinstance(blob_or_graph, STGraphBlob) else [blob_or_graph]


def _graph_labels(graph) -> torch.Tensor | None:
    if "y" in graph.dstdata:
        return graph.dstdata["y"]
    if "y" in graph.srcdata:
        return graph.srcdata["y"][: graph.num_dst_nodes]
    return None


class FlareEvolveGCN(nn.Module):
    def __init__(self, input_size: int, hidden_size: int, output_size: int = 1) -> None:
        super().__init__()
        self.initial_weight = nn.Parameter(torch.empty(input_size, hidden_size))
        nn.init.xavier_uniform_(self.initial_weight)
        self.mat_gru = MatGRUCell(in_feats=input_size, out_feats=hidden_size)
        self.pool_proj = nn.Linear(input_size, input_size)
        self.out = nn.Linear(hidden_size, output_size)

    def _pool_graph_context(self, graph) -> torch.Tensor:
        x = _graph_input(graph).float()[: graph.num_dst_nodes]
        return linear(x.mean(dim=0, keepdim=True), self.pool_proj.weight, self.pool_proj.bias)

    def forward(self, blob_or_graph, state: torch.Tensor | None = None):
        weights = self.initial_weight if state is None else state
        outputs = []
        for graph in _graph_sequence(blob_or_graph):
            weights = self.mat_gru(weights, self._pool_graph_context(graph))
            agg = _gcn_message_pass(graph, _graph_input(graph).float())
            h = linear(agg, weights.t().contiguous())
            outputs.append(linear(h, self.out.weight, self.out.bias))
        return (outputs if isinstance(blob_or_graph, STGraphBlob) else outputs[-1]), weights


class FlareTGCN(nn.Module):
    def __init__(self, input_size: int, hidden_size: int, output_size: int = 1) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.gcn = GCNStack(input_size, hidden_size * 3, num_layers=2)
        self.u_t = nn.Linear(hidden_size * 2, hidden_size)
        self.r_t = nn.Linear(hidden_size * 2, hidden_size)
        self.c_t = nn.Linear(hidden_size * 2, hidden_size)
        self.out = nn.Linear(hidden_size, output_size)

    def forward(self, blob_or_graph, state: torch.Tensor | None = None):
        outputs = []
        h = state
        for graph, urc in zip(_graph_sequence(blob_or_graph), self.gcn.layerwise(blob_or_graph)):
            h = graph.flare_fetch_state(h) if hasattr(graph, "flare_fetch_state") and h is not None else h
            if h is None:
                h = torch.zeros(urc.size(0), self.hidden_size, dtype=urc.dtype, device=urc.device)
            u, r, c = urc.chunk(3, dim=-1)
            h = rgru_cell(u, r, c, h, self.u_t.weight, self.u_t.bias, self.r_t.weight, self.r_t.bias,
                          self.c_t.weight, self.c_t.bias)
            if hasattr(graph, "flare_store_state"):
                graph.flare_store_state(h)
            outputs.append(linear(h, self.out.weight, self.out.bias))
        return (outputs if isinstance(blob_or_graph, STGraphBlob) else outputs[-1]), h


class FlareMPNNLSTM(nn.Module):
    def __init__(self, input_size: int, hidden_size: int, output_size: int = 1) -> None:
        super().__init__()
        self.hidden_size = hidden_size
        self.gcn = GCNStack(input_size, hidden_size, num_layers=2)
        self.rnn = nn.ModuleList([_LSTMCell(hidden_size, hidden_size), _LSTMCell(hidden_size, hidden_size)])
        self.out = nn.Linear(hidden_size, output_size)

    def forward(self, blob_or_graph, state=None):
        outputs = []
        h = state
        for graph, x in zip(_graph_sequence(blob_or_graph), self.gcn.layerwise(blob_or_graph)):
            h = graph.flare_fetch_state(h)
            s1 = None if h is None else h[0:2]
            s2 = None if h is None else h[2:4]
            x, _ = s1 = self.rnn[0](x, s1)
            x, _ = s2 = self.rnn[1](x, s2)
            h = tuple(s1) + tuple(s2)
            graph.flare_store_state(h)
            outputs.append(linear(x, self.out.weight, self.out.bias))
        return (outputs if isinstance(blob_or_graph, STGraphBlob) else outputs[-1]), h


@dataclass(frozen=True)
class FlareModelSpec:
    model_cls: type[nn.Module]


MODEL_SPECS: dict[str, FlareModelSpec] = {
    "evolvegcn": FlareModelSpec(FlareEvolveGCN),
    "tgcn": FlareModelSpec(FlareTGCN),
    "mpnn_lstm": FlareModelSpec(FlareMPNNLSTM),
    "gcn": FlareModelSpec(FlareTGCN),
}


def build_flare_model(model_name: str, input_size: int, hidden_size: int, output_size: int) -> nn.Module:
    key = model_name.lower()
    if key not in MODEL_SPECS:
        raise KeyError(f"Unsupported flare model: {model_name}")
    return MODEL_SPECS[key].model_cls(input_size=input_size, hidden_size=hidden_size, output_size=output_size)


def extract_graph_labels(blob_or_graph) -> torch.Tensor | None:
    graphs = _graph_sequence(blob_or_graph)
    if not graphs:
        return None
    y = _graph_labels(graphs[-1])
    if y is None:
        return None
    return y.view(-1, 1) if y.dim() == 1 else y
