"""Halo communication plan summarised from a partition's routes
(reference runtime/route/comm_plan.py, broken there)."""
from __future__ import annotations

from typing import Any


def plan_from_routes(routes: Any) -> dict[str, Any]:
    send = [sum(s) for s in routes.send_sizes]
    recv = [sum(r) for r in routes.recv_sizes]
    return {"snapshots": len(send), "send_rows": send, "recv_rows": recv,
            "max_send": max(send) if send else 0, "max_recv": max(recv) if recv else 0}
