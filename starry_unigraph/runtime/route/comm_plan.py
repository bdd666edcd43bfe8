"""Halo communication volume of a partition's snapshot routes (reference module
runtime/route/comm_plan.py, truncated there): rows sent and received per
snapshot, summarised for the session's runtime state."""
from __future__ import annotations

from typing import Any


def plan_from_routes(routes: Any) -> dict[str, Any]:
    """``routes``: a ``RouteData`` (per-snapshot send / receive size lists)."""
    send = [int(sum(s)) for s in routes.send_sizes]
    recv = [int(sum(r)) for r in routes.recv_sizes]
    return {"snapshots": len(send), "send_rows": send, "recv_rows": recv,
            "max_send": max(send, default=0), "max_recv": max(recv, default=0),
            "total_send": sum(send), "total_recv": sum(recv)}
