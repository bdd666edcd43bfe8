"""Worker for the multi-GPU DTDG test: MPNN-LSTM on a small synthetic snapshot
sequence, partitioned over the ranks, with the halo exchange and gradient
all-reduce over NVLink (comm.path p2p) or NCCL (comm.path nccl). Saves this
rank's losses and parameters.

    torchrun --nproc-per-node 2 tests/workers/dtdg_peer_worker.py --out DIR --path {p2p,nccl} [--decay]
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
    p.add_argument("--path", default="p2p", choices=["p2p", "nccl"])
    p.add_argument("--steps", type=int, default=6)
    p.add_argument("--decay", action="store_true", help="random chunk order + chunk_decay half (permuted rows)")
    a = p.parse_args()
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    from starry_unigraph import SchedulerSession
    from starry_unigraph.backends.dtdg.runtime.training import run_flare_train_step
    from starry_unigraph.distributed import finalize_distributed, initialize_distributed
    from starry_unigraph.ops import check_status

    cfg = {"model": {"name": "mpnn_lstm", "family": "mpnn_lstm", "task": "snapshot_node_regression",
                     "hidden_dim": 32, "window": {"size": 4}},
           "data": {"root": "./data", "name": "dtdg_peer", "format": "synthetic",
                    "synthetic": {"preset": "mpnn_lstm_large", "num_snapshots": 12, "num_nodes": 6000,
                                  "edges_per_snapshot": 40000, "feat_dim": 16}},
           "train": {"epochs": 1, "snaps": 12, "lr": 1e-3},
           "runtime": {"device": "cuda"},
           "dtdg": {"window_from_size": True, "chunk_order": "rand" if a.decay else None,
                    "chunk_decay": "half" if a.decay else None},
           "comm": {"path": a.path},
           "dist": {"backend": "nccl", "timeout_s": 120}}
    s = SchedulerSession.from_config(cfg)
    tag = f"{a.path}{'_decay' if a.decay else ''}"
    s.ctx.artifact_root = Path(a.out) / f"art_{tag}_w{world}_r{rank}"
    initialize_distributed(s.ctx.dist)
    s.prepare_data()
    s.build_runtime()
    losses = []
    for i, blob in enumerate(s.snapshot_core.iter_train(max_steps=a.steps)):
        out = run_flare_train_step(s.runtime, blob, {"meta": {}})
        losses.append(float(out["loss"]))
    torch.cuda.synchronize()
    check_status()
    flat = s.runtime.optimizer.flat.data.cpu()
    torch.save({"losses": losses, "params": flat, "halo": s.runtime.state.get("halo")},
               Path(a.out) / f"dtdg_{tag}_r{rank}.pt")
    from starry_unigraph.parallel.halo import set_halo_context

    set_halo_context(None)
    finalize_distributed(s.ctx.dist)
    print(json.dumps({"rank": rank, "losses": losses}), flush=True)


if __name__ == "__main__":
    main()
