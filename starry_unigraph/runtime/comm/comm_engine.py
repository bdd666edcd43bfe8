"""Communication engine of the unified runtime (reference runtime/comm/comm_engine.py:35-138,
a protocol there): asynchronous owner-routed exchange of node rows, delta push /
poll, remote fetch and gradient all-reduce with optional int8 compression
(one absmax scale shared by all ranks; int32 sums)."""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.distributed as dist
from torch import Tensor


@dataclass
class CommHandle:
    works: list[Any]
    result: Any

    def wait(self) -> Any:
        for w in self.works:
            w.wait()
        return self.result


def _world() -> int:
    return dist.get_world_size() if dist.is_available() and dist.is_initialized() else 1


class CommEngine:
    def __init__(self, owner: Tensor | None = None, rank: int = 0, int8_gradients: bool = False):
        self.owner = owner
        self.rank = rank
        self.int8_gradients = int8_gradients
        self._inbox: list[tuple[Tensor, Tensor]] = []

    def _a2a_rows(self, ids: Tensor, rows: Tensor, dest: Tensor) -> CommHandle:
        W = _world()
        if W == 1:
            return CommHandle([], (ids, rows))
        order = torch.argsort(dest, stable=True)
        ids, rows, dest = ids[order], rows[order], dest[order]
        sc_t = torch.bincount(dest, minlength=W)
        rc_t = torch.empty_like(sc_t)
        dist.all_to_all_single(rc_t, sc_t)
        sc, rc = sc_t.tolist(), rc_t.tolist()
        width = rows.size(1) if rows.dim() == 2 else 1
        r_ids = torch.empty(sum(rc), dtype=ids.dtype, device=ids.device)
        r_rows = torch.empty(sum(rc), width, dtype=rows.dtype, device=rows.device)
        w1 = dist.all_to_all_single(r_ids, ids.contiguous(), rc, sc, async_op=True)
        w2 = dist.all_to_all_single(r_rows.view(-1), rows.reshape(-1).contiguous(), [c * width for c in rc],
                                    [c * width for c in sc], async_op=True)
        return CommHandle([w1, w2], (r_ids, r_rows))

    def async_exchange(self, ids: Tensor, rows: Tensor) -> CommHandle:
        """Send each row to the owner of its id."""
        dest = self.owner[ids] if self.owner is not None else torch.zeros_like(ids)
        return self._a2a_rows(ids, rows, dest.to(ids.device))

    def push_delta(self, ids: Tensor, deltas: Tensor) -> None:
        self._inbox.append(self.async_exchange(ids, deltas).wait())

    def try_recv_delta(self) -> tuple[Tensor, Tensor] | None:
        return self._inbox.pop(0) if self._inbox else None

    def async_fetch(self, ids: Tensor, table: Tensor) -> CommHandle:
        """Request rows of ``ids`` from their owners and return them (two all-to-alls)."""
        W = _world()
        if W == 1:
            return CommHandle([], table[ids])
        dest = self.owner[ids].to(ids.device)
        req = self._a2a_rows(ids, ids.view(-1, 1).float(), dest).wait()[0]
        answer = table[req]
        back_dest = self.owner.new_zeros(req.numel())  # filled below
        # answer goes back to the requester: recompute requester ranks from the request counts
        sc_t = torch.bincount(dest, minlength=W)
        rc_t = torch.empty_like(sc_t)
        dist.all_to_all_single(rc_t, sc_t)
        back_dest = torch.repeat_interleave(torch.arange(W, device=ids.device), rc_t)
        order = torch.argsort(dest, stable=True)
        h = self._a2a_rows(req, answer, back_dest)
        r_ids, r_rows = h.wait()
        out = torch.empty(ids.numel(), table.size(1), dtype=table.dtype, device=table.device)
        out[order] = r_rows
        return CommHandle([], out)

    def all_reduce_gradients(self, params: list[torch.nn.Parameter]) -> None:
        W = _world()
        if W == 1:
            return
        grads = [p.grad for p in params if p.grad is not None]
        if not grads:
            return
        flat = torch.cat([g.reshape(-1) for g in grads])
        if self.int8_gradients:
            scale = flat.abs().max().clamp_min(1e-12) / 127.0
            dist.all_reduce(scale, op=dist.ReduceOp.MAX)
            q = torch.round(flat / scale).to(torch.int32)
            dist.all_reduce(q)
            flat = q.float() * scale
        else:
            dist.all_reduce(flat)
        flat /= W
        off = 0
        for g in grads:
            n = g.numel()
            g.copy_(flat[off:off + n].view_as(g))
            off += n
