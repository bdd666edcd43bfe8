"""Worker for the multi-GPU CTDG tests: trains a few TGN steps through the
public session API (one process per GPU under torchrun, or one process alone)
and saves the node tables, parameters and losses of this rank.

    python tests/workers/ctdg_peer_worker.py --out DIR --batch B --steps S --mode {hash,owner0} [--lr LR]

mode owner0: every node and every event belongs to rank 0 (other ranks see
empty batches, events assigned by owner), so rank 0 must reproduce a single-GPU
run with batch W*B. mode hash: nodes hash-partitioned, events assigned by
--assign (balanced: B events per rank; owner: the events of owned sources).
"""
import argparse
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--out", required=True)
    p.add_argument("--batch", type=int, default=100)
    p.add_argument("--steps", type=int, default=8)
    p.add_argument("--mode", default="hash", choices=["hash", "owner0"])
    p.add_argument("--lr", type=float, default=1e-3)
    p.add_argument("--graphs", type=int, default=1)
    p.add_argument("--assign", default="balanced", choices=["balanced", "owner"])
    p.add_argument("--sync", action="store_true", help="ctdg.async_sync false: each step waits for the write-backs")
    p.add_argument("--tag", default="", help="suffix of the output files")
    a = p.parse_args()
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    from starry_unigraph import SchedulerSession
    from starry_unigraph.ops import check_status

    cfg = {"model": {"name": "tgn", "family": "tgn", "task": "temporal_link_prediction", "hidden_dim": 32},
           "data": {"root": "./data", "name": "peer", "format": "synthetic",
                    "synthetic": {"preset": "tgn_cpu", "num_events": 6000, "edge_dim": 8, "num_src": 400,
                                  "num_dst": 120}},
           "train": {"epochs": 1, "batch_size": a.batch, "lr": a.lr},
           "runtime": {"device": "cuda", "cuda_graphs": bool(a.graphs)},
           "ctdg": {"mailbox_slots": 1, "dim_time": 16, "num_head": 2, "dropout": 0.0, "att_dropout": 0.0,
                    "event_partition": "owner" if a.mode == "owner0" else a.assign, "async_sync": not a.sync},
           "sampling": {"neighbor_limit": [5], "strategy": "recent", "history": 1},
           "graph": {"partition": "round_robin"},
           "dist": {"backend": "nccl", "timeout_s": 120}}
    s = SchedulerSession.from_config(cfg)
    s.ctx.artifact_root = Path(a.out) / f"art_w{world}_r{rank}{a.tag}"
    if world > 1:
        from starry_unigraph.distributed import initialize_distributed

        initialize_distributed(s.ctx.dist)
    s.prepare_data()
    if world > 1 and a.mode == "owner0":
        parts = s.prepared.directories.get("partitions", s.ctx.artifact_root / "partitions")
        n = int(torch.load(parts / "node_parts.pt").numel())
        e = int(torch.load(parts / "edge_parts.pt").numel())
        torch.save(torch.zeros(n, dtype=torch.long), parts / "node_parts.pt")
        torch.save(torch.zeros(e, dtype=torch.long), parts / "edge_parts.pt")
        s.prepared.provider_meta["max_local_batch"] = a.batch * world
    s.build_runtime()
    rt = s.ctdg_session.online_runtime
    losses, sizes = [], []
    for i, b in enumerate(rt.iter_batches("train", a.batch)):
        if i >= a.steps:
            break
        out = s.ctdg_session.train_step(b)
        losses.append(float(out["loss"]))
        sizes.append(b.size)
    torch.cuda.synchronize()
    check_status()
    mb = rt.memory
    eng = rt.engine
    torch.save({"memory": mb.memory.cpu(), "memory_ts": mb.memory_ts.cpu(), "mailbox": mb.mailbox.cpu(),
                "mailbox_ts": mb.mailbox_ts.cpu(), "params": eng.flat.data.cpu(), "losses": losses,
                "owner": mb.owner.cpu(), "peer": eng.peer is not None, "sizes": sizes},
               Path(a.out) / f"w{world}_r{rank}{a.tag}.pt")
    if world > 1:
        eng.reset_graphs()
        from starry_unigraph.distributed import finalize_distributed

        finalize_distributed(s.ctx.dist)
    print(json.dumps({"rank": rank, "steps": len(losses)}), flush=True)


if __name__ == "__main__":
    main()
