"""JSONL metrics log: one JSON object per line (step, split, loss, metrics,
timings). Rank 0 writes by default; every rank can write its own file with
``per_rank=True`` (file name gets ``.rank<r>``)."""
from __future__ import annotations

import json
import time
from pathlib import Path
from typing import Any


class MetricsLogger:
    def __init__(self, path: str | Path, rank: int = 0, per_rank: bool = False) -> None:
        self.rank = int(rank)
        p = Path(path)
        if per_rank:
            p = p.with_name(f"{p.name}.rank{self.rank}")
        self.path = p
        self.enabled = per_rank or self.rank == 0
        if self.enabled:
            self.path.parent.mkdir(parents=True, exist_ok=True)

    def log(self, **record: Any) -> None:
        if not self.enabled:
            return
        rec = {"time": time.time(), "rank": self.rank}
        rec.update({k: (float(v) if hasattr(v, "item") and getattr(v, "numel", lambda: 2)() == 1 else v)
                    for k, v in record.items()})
        with self.path.open("a") as f:
            f.write(json.dumps(rec, default=str) + "\n")

    def read(self) -> list[dict[str, Any]]:
        if not self.path.exists():
            return []
        return [json.loads(line) for line in self.path.read_text().splitlines() if line.strip()]
