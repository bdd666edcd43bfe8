"""CTDG feature route: owner-routed exchange of node rows between ranks
(reference backends/ctdg/runtime/route.py:19-217).

``exchange`` sends rows to the ranks that own them (all-to-all with counts)
and returns what this rank received; ``describe`` is written into the
artifacts (routes/manifest.json).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch


@dataclass
class AsyncExchangeHandle:
    works: list[Any]
    recv_ids: torch.Tensor
    recv_values: torch.Tensor

    def wait(self) -> tuple[torch.Tensor, torch.Tensor]:
        for w in self.works:
            w.wait()
        return self.recv_ids, self.recv_values


class CTDGFeatureRoute:
    def __init__(self, route_type: str = "all2all", world_size: int = 1):
        self.route_type = route_type
        self.world_size = int(world_size)

    def describe(self) -> dict[str, Any]:
        return {"route_type": self.route_type, "world_size": self.world_size, "type": "CTDGFeatureRoute"}

    def exchange(self, ids: torch.Tensor, values: torch.Tensor, owner: torch.Tensor,
                 async_op: bool = False) -> AsyncExchangeHandle | tuple[torch.Tensor, torch.Tensor]:
        import torch.distributed as dist

        if self.world_size == 1 or not dist.is_initialized():
            h = AsyncExchangeHandle([], ids, values)
            return h if async_op else h.wait()
        order = torch.argsort(owner, stable=True)
        ids, values = ids[order], values[order]
        sc_t = torch.bincount(owner[order], minlength=self.world_size)
        rc_t = torch.empty_like(sc_t)
        dist.all_to_all_single(rc_t, sc_t)
        sc, rc = sc_t.tolist(), rc_t.tolist()
        width = values[0].numel() if values.numel() else (values.size(1) if values.dim() == 2 else 1)
        r_ids = torch.empty(sum(rc), dtype=ids.dtype, device=ids.device)
        r_vals = torch.empty(sum(rc), width, dtype=values.dtype, device=values.device)
        w1 = dist.all_to_all_single(r_ids, ids.contiguous(), rc, sc, async_op=True)
        w2 = dist.all_to_all_single(r_vals.view(-1), values.reshape(-1).contiguous(), [c * width for c in rc],
                                    [c * width for c in sc], async_op=True)
        h = AsyncExchangeHandle([w1, w2], r_ids, r_vals)
        return h if async_op else h.wait()
