"""CTDG partitioning (reference backends/ctdg/preprocess_partition.py:18-245).

* round-robin node ownership (``id % num_parts``, a hash partition),
* edge ownership = partition of the event's source node,
* SPEED: the reference shells out to an external ``starrygl_partition``
  binary (not part of the repository); the same hook is kept: when the binary
  is given via ``ctdg.speed_binary`` / ``$SPEED_PARTITION_BIN`` it is run with
  the reference's text I/O, otherwise the caller falls back to round-robin.
"""
from __future__ import annotations

import os
import subprocess
import tempfile
from pathlib import Path
from typing import Any

import torch


def build_round_robin_node_parts(num_nodes: int, num_parts: int) -> torch.Tensor:
    return torch.arange(num_nodes, dtype=torch.long) % max(1, num_parts)


def derive_edge_parts(src: torch.Tensor, node_parts: torch.Tensor) -> torch.Tensor:
    return node_parts[src.long()].long()


def speed_partition(dataset: Any, num_parts: int, config: dict[str, Any] | None = None):
    cfg = (config or {}).get("ctdg", {})
    binary = cfg.get("speed_binary") or os.environ.get("SPEED_PARTITION_BIN")
    if not binary or not Path(binary).exists():
        raise FileNotFoundError("SPEED partitioner binary not available")
    with tempfile.TemporaryDirectory() as tmp:
        inp, out = Path(tmp) / "edges.txt", Path(tmp) / "parts.txt"
        with inp.open("w") as f:
            for s, d, t in zip(dataset.src.tolist(), dataset.dst.tolist(), dataset.ts.tolist()):
                f.write(f"{s} {d} {t}\n")
        cmd = [str(binary), str(inp), str(out), str(num_parts), str(cfg.get("speed_beta", 1.0)),
               str(cfg.get("speed_topk_type", "decay")), str(cfg.get("speed_topk_ratio", 0.01)),
               str(cfg.get("speed_reorder_type", "normal"))]
        subprocess.run(cmd, check=True, timeout=3600)
        parts = torch.zeros(dataset.num_nodes, dtype=torch.long)
        for line in out.read_text().splitlines():
            if line.strip():
                n, p = line.split()[:2]
                parts[int(n)] = int(p)
    return parts, derive_edge_parts(dataset.src, parts)
