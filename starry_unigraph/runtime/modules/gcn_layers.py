"""Multi-layer GCN over partitioned snapshot blocks
(reference runtime/modules/gcn_layers.py:20-165).

Per layer: normalised neighbour aggregation and ``Linear(bias=False)``, ReLU
between layers. For a block, the first layer aggregates the stored source
features (local rows + halo rows), then applies its linear map. Later layers
exchange halo rows (the block's ``Route`` over NCCL, or peer memory over
NVLink, when running distributed; zero rows otherwise) and run their linear
map first: A (H W^T) = (A H) W^T without a bias, so the exchanged rows are the
layer's output width and, on the NVLink path, the GEMM's epilogue writes them
straight into the staging buffer the peers read (``parallel/halo_linear.py``).
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn as nn

from starry_unigraph.ops.dtdg import gcn_aggregate, linear


def _graph_sequence(blob_or_graph):
    if hasattr(blob_or_graph, "__iter__") and not hasattr(blob_or_graph, "edge_src"):
        return list(blob_or_graph)
    return [blob_or_graph]


def _graph_input(graph) -> torch.Tensor:
    if "x" in graph.dstdata:
        return graph.dstdata["x"]
    return graph.srcdata["x"]


def _gcn_norm(graph) -> torch.Tensor:
    return graph.edge_norm().unsqueeze(-1)


def _gcn_message_pass(graph, x: torch.Tensor, exchange: bool | None = None) -> torch.Tensor:
    """Normalised neighbour sum of `graph` over source rows built from `x`.

    `x` is either the block's stored source features (local + halo rows, nothing
    to exchange) or a layer output over the block's destination rows, whose halo
    rows are fetched from their owners (``exchange``). When not given,
    ``exchange`` is inferred from the row count; callers that know which case
    they are in pass it, since a block without halo rows has equal counts and
    every rank must still take part in the exchange."""
    if exchange is None:
        exchange = x.size(0) != graph.num_src_nodes
    if not exchange:
        if x.size(0) != graph.num_src_nodes:
            raise ValueError(f"Unexpected feature rows for block graph: got {x.size(0)}, expected "
                             f"{graph.num_src_nodes} source rows")
        return gcn_aggregate(graph, x)
    if x.size(0) != graph.num_dst_nodes:
        raise ValueError(f"Unexpected feature rows for block graph: got {x.size(0)}, expected "
                         f"{graph.num_dst_nodes} destination rows")
    route = getattr(graph, "route", None)
    if route is not None and route.send_index is not None and dist.is_available() and dist.is_initialized():
        from starry_unigraph.parallel.halo import get_halo_context, halo_aggregate

        hc = get_halo_context()
        if x.is_cuda and hc is not None and hc.supports(int(x.size(-1))):  # halo rows pulled from the peers
            return halo_aggregate(graph, x)
        return gcn_aggregate(graph, route.forward(x))
    extra = graph.num_src_nodes - graph.num_dst_nodes  # no route: halo rows read as zeros
    src_x = torch.cat([x, x.new_zeros(extra, x.size(-1))], dim=0) if extra > 0 else x
    return gcn_aggregate(graph, src_x)


def _linear_then_exchange(graph, x: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """Normalised neighbour sum of `graph` over the rows of x W^T, whose halo rows
    come from their owners. On the NVLink path (an active halo context that takes
    the width) one fused layer; otherwise the linear map, then the message pass."""
    route = getattr(graph, "route", None)
    if (x.is_cuda and route is not None and route.send_index is not None and dist.is_available()
            and dist.is_initialized()):
        from starry_unigraph.parallel.halo import get_halo_context

        hc = get_halo_context()
        if hc is not None and int(weight.size(0)) % 4 == 0 and hc.supports(int(weight.size(0))):
            from starry_unigraph.parallel.halo_linear import halo_linear_aggregate

            return halo_linear_aggregate(graph, x, weight, hc)
    return _gcn_message_pass(graph, linear(x, weight, None, 0), exchange=True)


class GCNStack(nn.Module):
    def __init__(self, input_size: int, hidden_size: int, num_layers: int = 2) -> None:
        super().__init__()
        self.layers = nn.ModuleList()
        d = input_size
        for _ in range(num_layers):
            self.layers.append(nn.Linear(d, hidden_size, bias=False))
            d = hidden_size

    def forward_graph(self, graph, x: torch.Tensor | None = None) -> torch.Tensor:
        h = _graph_input(graph) if x is None else x
        last = len(self.layers) - 1
        for i, layer in enumerate(self.layers):
            act = 1 if i < last else 0
            if i > 0 or x is not None:
                # input over the destination rows only: linear map first, then the exchange
                h = _linear_then_exchange(graph, h.float(), layer.weight)
                if act:
                    h = torch.relu(h)
            else:
                # the block's stored source rows (halo rows included when the block has any)
                h = _gcn_message_pass(graph, h.float(), exchange=None)
                h = linear(h, layer.weight, None, act)
        return h

    def layerwise(self, blob_or_graph) -> list[torch.Tensor]:
        return [self.forward_graph(g) for g in _graph_sequence(blob_or_graph)]
