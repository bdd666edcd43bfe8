"""Reference arm of bench.py: the unmodified reference package (installed under
baseline/_ref) driven through its own public API on the headline workload.

    python bench_reference.py --data DIR --name NAME --steps K --warmup W [--batch B]

Run by ``bench.py --impl reference`` in a subprocess whose import path holds
only baseline/_ref (working directory outside this repository), so the
reference's ``starry_unigraph`` package is the one imported. The event stream
(BASELINE.json config 3 shape) is written beforehand by bench.py into
DIR/NAME/{edges.csv, edge_features.pt}, the reference's CSV format
(data/raw_temporal.py _load_from_ctdg_csv). The steps are the reference's stock
``SchedulerSession.ctdg_session.train_step`` calls (backends/ctdg/runtime/
runtime.py train_step), timed on the device with CUDA events after W untimed
steps, max over ranks. Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

# the reference's package must be the one imported: drop this repository from the path
_HERE = os.path.dirname(os.path.abspath(__file__))
sys.path[:] = [q for q in sys.path if os.path.abspath(q or os.getcwd()) != _HERE]


def main() -> int:
    p = argparse.ArgumentParser()
    p.add_argument("--data", required=True)
    p.add_argument("--name", required=True)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--batch", type=int, default=600)
    a = p.parse_args()
    import torch
    import torch.distributed as dist
    from starry_unigraph import SchedulerSession  # the reference's package (baseline/_ref)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    cfg = {
        "model": {"name": "tgn", "family": "tgn", "task": "temporal_link_prediction", "hidden_dim": 100},
        "data": {"root": a.data, "name": a.name, "format": "auto"},
        "train": {"epochs": 1, "batch_size": a.batch, "lr": 1e-4},
        "runtime": {"device": "cuda"},
        "ctdg": {"mailbox_slots": 1, "dim_time": 100, "num_head": 2, "dropout": 0.1, "att_dropout": 0.1,
                 "async_sync": True},
        "sampling": {"neighbor_limit": [10], "strategy": "recent", "history": 1},
        "graph": {"partition": "round_robin"},
        "dist": {"backend": "nccl"},
    }
    session = SchedulerSession.from_config(cfg)
    if world > 1 and not dist.is_initialized():
        from starry_unigraph.distributed import initialize_distributed

        initialize_distributed(session.ctx.dist)
    session.prepare_data()
    session.build_runtime()
    batches = []
    for b in session.ctdg_session.iter_train(session.ctx):
        batches.append(b)
        if len(batches) >= a.warmup + a.steps:
            break
    for b in batches[: a.warmup]:
        session.ctdg_session.train_step(b)
    timed = batches[a.warmup: a.warmup + a.steps]
    events = float(sum(int(b.src.numel()) for b in timed))
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    t0 = time.perf_counter()
    for b in timed:
        session.ctdg_session.train_step(b)
    end.record()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    stats = torch.tensor([start.elapsed_time(end), wall, events], dtype=torch.float64, device="cuda")
    if world > 1:
        mx = stats[:2].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        ev = stats[2:].clone()
        dist.all_reduce(ev)
        stats = torch.cat([mx, ev])
    dev_ms, wall_s, events_all = stats.tolist()
    if rank == 0:
        print(json.dumps({"impl": "reference", "metric": "TGN train events/sec", "value": events_all / (dev_ms / 1e3),
                          "unit": "events/s", "n_gpus": world, "steps": len(timed), "warmup": a.warmup,
                          "ms_per_step": dev_ms / max(1, len(timed)), "higher_is_better": True, "scaling": "weak",
                          "dtype": "fp32", "data": "synthetic (random-init weights)",
                          "e2e": {"value": events_all / wall_s, "unit": "events/s"},
                          "config": {"model": "TGN (1-layer temporal attention, 2 heads), CTDG online + async_sync",
                                     "global_batch": a.batch * world, "parallelism": f"dp{world}+memory-partition"}}),
              flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
