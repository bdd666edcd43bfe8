"""Communication plans (reference module runtime/route/comm_plan.py, truncated
there): the halo volume of a partition's snapshot routes, rows sent and
received per snapshot, summarised for the session's runtime state; and the
spatial / state dependence declarations of a chunk."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any

import torch

from starry_unigraph.data.partition import RouteData  # noqa: F401  (the reference keeps a copy here)


def plan_from_routes(routes: Any) -> dict[str, Any]:
    """``routes``: a ``RouteData`` (per-snapshot send / receive size lists)."""
    send = [int(sum(s)) for s in routes.send_sizes]
    recv = [int(sum(r)) for r in routes.recv_sizes]
    return {"snapshots": len(send), "send_rows": send, "recv_rows": recv,
            "max_send": max(send, default=0), "max_recv": max(recv, default=0),
            "total_send": sum(send), "total_recv": sum(recv)}


# ---------------------------------------------------------------------------
# Chunk dependence declarations (reference runtime/route/comm_plan.py:9-27 and
# 175-188, where StateDeps.stale_filter is cut off mid-statement)
# ---------------------------------------------------------------------------
@dataclass
class SpatialDeps:
    """A chunk's spatial dependence: how many embedding rows it sends to and
    receives from every (rank, cluster) pair of the same time slice.

    ``send_sizes`` / ``recv_sizes`` are indexed by ``rank * num_clusters +
    cluster``; ``send_index`` (optional) lists the global node id of every row
    to send, cluster after cluster, ``send_index_ptr`` its offsets per cluster."""

    send_sizes: torch.Tensor
    recv_sizes: torch.Tensor
    send_index: torch.Tensor | None = None
    send_index_ptr: torch.Tensor | None = None

    def to_route(self, chunks, in_chunks=None, num_clusters: int | None = None, world_size: int | None = None):
        """The halo ``Route`` of the clusters `chunks` (ids inside each rank):
        per rank the rows of those clusters; the send index of the clusters
        `in_chunks` (default: `chunks`) when the dependence carries one."""
        from starry_unigraph.runtime.route.route import Route

        chunks = torch.as_tensor(chunks, dtype=torch.long).view(-1)
        send, recv = torch.as_tensor(self.send_sizes).view(-1), torch.as_tensor(self.recv_sizes).view(-1)
        if num_clusters is None:
            num_clusters = int(send.numel() // max(1, world_size or 1))
        if world_size is None:
            world_size = int(send.numel() // max(1, num_clusters))
        send_sizes = [int(send[r * num_clusters + chunks].sum()) for r in range(world_size)]
        recv_sizes = [int(recv[r * num_clusters + chunks].sum()) for r in range(world_size)]
        index = None
        if self.send_index is not None and self.send_index_ptr is not None:
            sel = chunks if in_chunks is None else torch.as_tensor(in_chunks, dtype=torch.long).view(-1)
            ptr = torch.as_tensor(self.send_index_ptr, dtype=torch.long)
            index = torch.cat([self.send_index[int(ptr[c]):int(ptr[c + 1])] for c in sel.tolist()]) \
                if sel.numel() else self.send_index[:0]
        return Route(send_sizes, recv_sizes, index)


@dataclass
class StateDeps:
    """A chunk's state dependence: the remote nodes whose memory it reads (with
    the cluster that owns each) and its local nodes whose new memory other
    clusters read (with, per node, the clusters to notify)."""

    read_boundary: torch.Tensor
    read_from_cluster: torch.Tensor
    write_notify: torch.Tensor
    write_to_clusters: list = field(default_factory=list)

    def stale_filter(self, mask: torch.Tensor) -> "StateDeps":
        """Keep only the write notifications where `mask` is true (e.g. the rows
        whose memory changed enough to be worth sending); reads are unchanged."""
        mask = torch.as_tensor(mask, dtype=torch.bool).view(-1)
        keep = torch.nonzero(mask).view(-1).tolist()
        clusters = [self.write_to_clusters[i] for i in keep] if self.write_to_clusters else []
        return StateDeps(self.read_boundary, self.read_from_cluster, self.write_notify[mask], clusters)
