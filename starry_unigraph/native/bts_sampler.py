"""Python face of the host temporal-neighbour sampler in ``starry_unigraph._native``
(reference interface: native/bts_sampler.py:11-85).

``build_temporal_neighbor_block`` builds (or fetches, by graph name) the native
T-CSR; ``BTSNativeSampler`` wraps a native ``ParallelSampler`` over it. The native
object is created on first use, and every tensor handed to it is normalised to
the contiguous CPU dtype the C++ side reads (int64 ids and timestamps, fp32
weights, int32 partition maps), so callers may pass device tensors or narrower
integer types.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from starry_unigraph.lib import load_bts_sampler_module

SAMPLER_POLICIES = ("recent", "uniform", "weighted", "boundery_recent_uniform", "boundery_recent_decay")


def _host(t: torch.Tensor | None, dtype: torch.dtype) -> torch.Tensor | None:
    return None if t is None else t.detach().to(device="cpu", dtype=dtype).contiguous()


def is_bts_sampler_available() -> bool:
    try:
        load_bts_sampler_module()
        return True
    except Exception:  # noqa: BLE001 - any import failure means "not available"
        return False


def build_temporal_neighbor_block(graph_name: str, row: torch.Tensor, col: torch.Tensor, num_nodes: int,
                                  eid: torch.Tensor, edge_weight: torch.Tensor | None = None,
                                  timestamp: torch.Tensor | None = None, is_distinct: int = 0):
    """Native T-CSR of the events (row -> col), keyed by ``col``, cached by name."""
    native = load_bts_sampler_module()
    return native.get_neighbors(graph_name, _host(row, torch.long), _host(col, torch.long), int(num_nodes),
                                int(is_distinct), _host(eid, torch.long), None, _host(edge_weight, torch.float32),
                                _host(timestamp, torch.long))


@dataclass(frozen=True)
class _SamplerSpec:
    num_nodes: int
    num_edges: int
    num_layers: int
    fanout: tuple[int, ...]
    workers: int
    policy: str
    local_part: int
    probability: float


class BTSNativeSampler:
    """Multi-layer temporal sampler over a native T-CSR ``tnb``."""

    def __init__(self, tnb: Any, num_nodes: int, num_edges: int, num_layers: int, fanout: list[int],
                 workers: int = 1, policy: str = "uniform", local_part: int = -1,
                 edge_part: torch.Tensor | None = None, node_part: torch.Tensor | None = None,
                 probability: float = 1.0) -> None:
        if policy not in SAMPLER_POLICIES:
            raise ValueError(f"unknown sampling policy {policy!r} (one of {SAMPLER_POLICIES})")
        self.tnb = tnb
        self.spec = _SamplerSpec(int(num_nodes), int(num_edges), int(num_layers), tuple(int(f) for f in fanout),
                                 max(1, int(workers)), str(policy), int(local_part), float(probability))
        # partition maps (all zeros: every node and event in partition 0)
        self.edge_part = torch.zeros(self.spec.num_edges, dtype=torch.int32) if edge_part is None \
            else _host(edge_part, torch.int32)
        self.node_part = torch.zeros(self.spec.num_nodes, dtype=torch.int32) if node_part is None \
            else _host(node_part, torch.int32)
        self._native = None

    def __getattr__(self, name: str) -> Any:  # num_nodes, fanout, policy, ... read through the spec
        spec = self.__dict__.get("spec")
        if spec is not None and name in _SamplerSpec.__dataclass_fields__:
            value = getattr(spec, name)
            return list(value) if name == "fanout" else value
        raise AttributeError(name)

    def _sampler(self):
        if self._native is None:
            s = self.spec
            self._native = load_bts_sampler_module().ParallelSampler(
                self.tnb, s.num_nodes, s.num_edges, s.workers, list(s.fanout), s.num_layers, s.policy,
                s.local_part, self.edge_part, self.node_part, s.probability)
        return self._native

    def sample_from_nodes(self, nodes: torch.Tensor, ts: torch.Tensor | None = None):
        """Sample around `nodes` at times `ts` (time 0 when omitted); returns the
        native per-layer blocks."""
        roots = _host(nodes, torch.long)
        times = torch.zeros(roots.numel(), dtype=torch.long) if ts is None else _host(ts, torch.long)
        native = self._sampler()
        native.neighbor_sample_from_nodes(roots, times, None)
        return native.get_ret()

    def reset(self) -> None:
        if self._native is not None:
            self._native.reset()
