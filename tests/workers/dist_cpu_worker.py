"""Worker for the multi-process CPU tests (gloo): one epoch through the public
session API on mock data, then this rank's parameters, losses and outcome are
saved. Launched by torchrun with --nproc-per-node 2.

    python -m torch.distributed.run --nproc-per-node 2 ... dist_cpu_worker.py --family F --out DIR
"""
import argparse
import json
import os
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--family", default="mpnn_lstm")
    p.add_argument("--out", required=True)
    p.add_argument("--timeout", type=float, default=60.0)
    p.add_argument("--heartbeat", type=float, default=0.0)
    a = p.parse_args()
    import torch

    from starry_unigraph import SchedulerSession
    from starry_unigraph.distributed import finalize_distributed, initialize_distributed

    rank = int(os.environ["RANK"])
    ctdg = a.family in ("tgn", "jodie", "dyrep", "tgat", "apan")
    cfg = {"model": {"name": a.family, "family": a.family,
                     "task": "temporal_link_prediction" if ctdg else "snapshot_node_regression", "hidden_dim": 16},
           "data": {"root": str(Path(a.out) / "data"), "name": f"dist_{a.family}", "format": "mock"},
           "train": {"epochs": 1, "batch_size": 8, "snaps": 12},
           "runtime": {"device": "cpu"},
           "graph": {"storage": "events" if ctdg else "snapshots"},
           "ctdg": {"dim_time": 8, "mailbox_slots": 1},
           "dist": {"backend": "gloo", "timeout_s": a.timeout, "heartbeat_s": a.heartbeat}}
    s = SchedulerSession.from_config(cfg)
    s.ctx.artifact_root = Path(a.out) / f"art_r{rank}"
    initialize_distributed(s.ctx.dist)
    t0 = time.time()
    outcome = {"rank": rank, "error": None}
    try:
        s.prepare_data()
        s.build_runtime()
        r = s.run_epoch("train")
        outcome["steps"] = r["steps"]
        outcome["loss"] = r["loss"]
        model = s.runtime.model.module if hasattr(s.runtime.model, "module") else s.runtime.model
        torch.save({"params": [p.detach().clone() for p in model.parameters()], "losses":
                    [o.get("loss") for o in r["outputs"] if isinstance(o.get("loss"), float)]},
                   Path(a.out) / f"r{rank}.pt")
    except Exception as exc:  # the failure-detection test expects the survivors to land here
        outcome["error"] = type(exc).__name__
        outcome["message"] = str(exc)[:500]
    outcome["elapsed_s"] = time.time() - t0
    (Path(a.out) / f"outcome_r{rank}.json").write_text(json.dumps(outcome))
    if outcome["error"] is None:
        finalize_distributed(s.ctx.dist)
    os._exit(0 if outcome["error"] is None else 3)


if __name__ == "__main__":
    main()
