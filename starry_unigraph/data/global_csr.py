"""Global temporal CSR protocol (reference data/global_csr.py:15-76) backed by
the T-CSR of the CTDG sampler."""
from __future__ import annotations

from typing import Protocol

import torch
from torch import Tensor


class GlobalCSR(Protocol):
    def neighbors(self, node: int) -> tuple[Tensor, Tensor, Tensor]: ...

    def slice_time(self, t0: float, t1: float) -> "GlobalCSR": ...


class TemporalGlobalCSR:
    def __init__(self, src: Tensor, dst: Tensor, ts: Tensor, num_nodes: int, eid: Tensor | None = None):
        from starry_unigraph.backends.ctdg.runtime.sampler import TemporalCSR

        self.src, self.dst, self.ts = src.long(), dst.long(), ts
        self.eid = torch.arange(src.numel()) if eid is None else eid.long()
        self.num_nodes = int(num_nodes)
        self.csr = TemporalCSR.build(self.src, self.dst, self.eid, ts.long(), self.num_nodes)

    def neighbors(self, node: int) -> tuple[Tensor, Tensor, Tensor]:
        a, b = int(self.csr.rowptr[node]), int(self.csr.rowptr[node + 1])
        return self.csr.nbr[a:b], self.csr.ts[a:b], self.csr.eid[a:b]

    def slice_time(self, t0: float, t1: float) -> "TemporalGlobalCSR":
        m = (self.ts >= t0) & (self.ts < t1)
        return TemporalGlobalCSR(self.src[m], self.dst[m], self.ts[m], self.num_nodes, self.eid[m])
