"""Differentiable halo exchange for partitioned snapshots
(reference backends/dtdg/runtime/route.py:28-350).

``Route`` describes, for one snapshot on one partition, which local rows are
sent to which peer (``send_index`` grouped by peer, ``send_sizes``) and how
many halo rows arrive from each peer (``recv_sizes``). ``forward(x)`` returns
``[x ; received halo rows]``; its backward sends the halo-row gradients back
and scatter-adds them into the owners' rows.

``Route.forward`` is the collective transport (``all_to_all_single``, the
reference's; the baseline). With ``comm.path: p2p`` on CUDA the GCN layers do
not call it: ``starry_unigraph.parallel.halo.halo_aggregate`` reads the halo
rows from the owners' memory inside the aggregation kernel and pushes their
gradients back with remote atomic adds.

``Route.from_graph`` partitions a global edge list into per-partition blocks
(edges owned by the destination's partition, halo = remote sources).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch
import torch.autograd as autograd
import torch.distributed as dist

from starry_unigraph.data.partition import EID, NID, SnapshotBlock

_TRANSPORT = {"path": "nccl"}


def set_route_transport(path: str) -> None:
    _TRANSPORT["path"] = str(path)


@dataclass
class Route:
    send_sizes: list[int]
    recv_sizes: list[int]
    send_index: torch.Tensor | None = None
    group: Any = None

    @property
    def send_len(self) -> int:
        return int(sum(self.send_sizes))

    @property
    def recv_len(self) -> int:
        return int(sum(self.recv_sizes))

    def forward(self, x: torch.Tensor, reverse: bool = False, group: Any = None) -> torch.Tensor:
        if self.send_index is None:
            return x
        return RouteExchange.apply(x, self, reverse, self.group if group is None else group)

    def pin_memory(self, device: str | None = None) -> "Route":
        return Route(self.send_sizes, self.recv_sizes,
                     None if self.send_index is None else self.send_index.pin_memory(), self.group)

    def to(self, device=None, dtype=None, non_blocking: bool = False, copy: bool = False) -> "Route":
        return Route(self.send_sizes, self.recv_sizes,
                     None if self.send_index is None else self.send_index.to(device=device, non_blocking=non_blocking),
                     self.group)

    def describe(self) -> dict[str, Any]:
        return {"parts": len(self.send_sizes), "send_len": self.send_len, "recv_len": self.recv_len,
                "send_sizes": [int(s) for s in self.send_sizes], "recv_sizes": [int(s) for s in self.recv_sizes],
                "has_send_index": self.send_index is not None,
                "active_recv_parts": [i for i, s in enumerate(self.recv_sizes) if int(s) > 0]}

    @classmethod
    def from_empty(cls, num_nodes: int, edge_index: torch.Tensor) -> list[SnapshotBlock]:
        blk = SnapshotBlock(num_src_nodes=num_nodes, num_dst_nodes=num_nodes, edge_src=edge_index[0].long(),
                            edge_dst=edge_index[1].long())
        ids = torch.arange(num_nodes, dtype=torch.long)
        blk.srcdata[NID] = ids
        blk.dstdata[NID] = ids
        blk.edata[EID] = torch.arange(edge_index.size(1), dtype=torch.long)
        return [blk]

    @classmethod
    def from_graph(cls, node_parts: torch.Tensor | int, edge_index: torch.Tensor,
                   num_parts: int | None = None) -> list[SnapshotBlock]:
        if not isinstance(node_parts, torch.Tensor):
            return cls.from_empty(int(node_parts), edge_index)
        node_parts = node_parts.long()
        if num_parts is None:
            num_parts = int(node_parts.max()) + 1 if node_parts.numel() else 1
        num_parts = max(1, int(num_parts))
        src_all, dst_all = edge_index[0].long(), edge_index[1].long()
        dst_part = node_parts[dst_all]
        src_part = node_parts[src_all]
        order = torch.argsort(dst_part, stable=True)
        bounds = torch.searchsorted(dst_part[order], torch.arange(num_parts + 1))
        dst_ids_list, edge_ids_list, recv_lists = [], [], []
        for p in range(num_parts):
            dst_ids = torch.nonzero(node_parts == p).view(-1)
            eids = order[bounds[p]:bounds[p + 1]]
            remote = src_all[eids][src_part[eids] != p]
            halo = torch.unique(remote)                       # sorted ids of remote sources
            halo_part = node_parts[halo]
            horder = torch.argsort(halo_part, stable=True)    # grouped by owning partition
            halo = halo[horder]
            recv_lists.append([halo[halo_part[horder] == q] for q in range(num_parts)])
            dst_ids_list.append(dst_ids)
            edge_ids_list.append(eids)
        xmap = torch.empty(node_parts.numel(), dtype=torch.long)
        blocks: list[SnapshotBlock] = []
        for p in range(num_parts):
            dst_ids = dst_ids_list[p]
            remote = torch.cat(recv_lists[p])
            src_ids = torch.cat([dst_ids, remote])
            xmap[src_ids] = torch.arange(src_ids.numel())
            send_ids = [recv_lists[q][p] for q in range(num_parts)]   # rows of p that q needs
            send_cat = torch.cat(send_ids)
            # send_index addresses p's local rows: map through p's own dst ordering
            loc = torch.empty(node_parts.numel(), dtype=torch.long)
            loc[dst_ids] = torch.arange(dst_ids.numel())
            send_index = loc[send_cat] if send_cat.numel() else torch.zeros(0, dtype=torch.long)
            eids = edge_ids_list[p]
            blk = SnapshotBlock(num_src_nodes=int(src_ids.numel()), num_dst_nodes=int(dst_ids.numel()),
                                edge_src=xmap[src_all[eids]], edge_dst=xmap[dst_all[eids]])
            blk.srcdata[NID] = src_ids
            blk.dstdata[NID] = dst_ids
            blk.edata[EID] = eids
            blk.route = cls(send_sizes=[int(t.numel()) for t in send_ids],
                            recv_sizes=[int(t.numel()) for t in recv_lists[p]], send_index=send_index)
            blocks.append(blk)
        return blocks


def _a2a(out: torch.Tensor, inp: torch.Tensor, out_sizes: list[int], in_sizes: list[int], group: Any) -> None:
    dist.all_to_all_single(out, inp, out_sizes, in_sizes, group=group)


class RouteExchange(autograd.Function):
    """forward: [x ; halo] ; backward: grad_x + scatter_add(send_index, returned halo grads)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, route: Route, reverse: bool, group: Any):
        if not dist.is_available() or not dist.is_initialized():
            raise RuntimeError("torch.distributed must be initialized before using Route.forward")
        ctx.route, ctx.reverse, ctx.group = route, reverse, group
        send = x.detach()[route.send_index]
        recv = torch.empty(route.recv_len, *x.shape[1:], dtype=x.dtype, device=x.device)
        _a2a(recv, send.contiguous(), route.recv_sizes, route.send_sizes, group)
        return torch.cat([x.detach(), recv], dim=0)

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        route = ctx.route
        n_local = grad.size(0) - route.recv_len
        gx = grad[:n_local].clone()
        back = torch.empty(route.send_len, *grad.shape[1:], dtype=grad.dtype, device=grad.device)
        _a2a(back, grad[n_local:].contiguous(), route.send_sizes, route.recv_sizes, ctx.group)
        if back.numel():
            gx.index_add_(0, route.send_index, back)
        return gx, None, None, None
