"""Train, validate and test a DTDG model (mpnn_lstm, tgcn, evolvegcn, gcn) through
``SchedulerSession``: the Flare pipeline over a snapshot sequence, nodes partitioned over
the ranks of one node.

    python examples/train_mpnn_lstm.py --config configs/mpnn_lstm_nvlink.yaml
    python examples/train_mpnn_lstm.py --config configs/tgcn_large.yaml --nodes 200000 --edges 2000000
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 4 --master-addr 127.0.0.1 \
        --master-port 29500 examples/train_mpnn_lstm.py --config configs/mpnn_lstm_nvlink.yaml

Every epoch prints (rank 0) the train and validation losses (the mean over all ranks' nodes,
the summary's ``global_loss``) and the training throughput in
snapshots per second (training windows per second, the slowest rank's time). Rank 0 writes
the checkpoint of the epoch with the lowest validation loss to ``runtime.checkpoint``; the
test phase loads it and reports MAE / RMSE / NMAE for regression tasks, accuracy for
classification tasks.

Reference counterparts: examples/train_mpnn_lstm_4gpu.py and examples/bench_mpnn_lstm.py of
the reference.
"""
from __future__ import annotations

import argparse
import math
import os
import sys
import time
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def _args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--config", default=str(Path(__file__).resolve().parents[1] / "configs" / "mpnn_lstm_nvlink.yaml"))
    p.add_argument("--mode", default="all", choices=["prepare", "train", "test", "all"])
    p.add_argument("--artifact-root", default=None)
    p.add_argument("--epochs", type=int, default=None)
    p.add_argument("--lr", type=float, default=None)
    p.add_argument("--device", default=None, help="cpu | cuda")
    p.add_argument("--backend", default=None, help="process-group backend: nccl (GPUs) | gloo (CPU ranks)")
    p.add_argument("--snapshots", type=int, default=None, help="synthetic sequences: number of snapshots")
    p.add_argument("--nodes", type=int, default=None, help="synthetic sequences: number of nodes")
    p.add_argument("--edges", type=int, default=None, help="synthetic sequences: edges per snapshot")
    return p.parse_args(argv)


def _overrides(a: argparse.Namespace) -> dict:
    o: dict = {}
    for key, val in (("epochs", a.epochs), ("lr", a.lr)):
        if val is not None:
            o.setdefault("train", {})[key] = val
    if a.device is not None:
        o.setdefault("runtime", {})["device"] = a.device
    if a.backend is not None:
        o.setdefault("dist", {})["backend"] = a.backend
    syn = {k: int(v) for k, v in (("num_snapshots", a.snapshots), ("num_nodes", a.nodes),
                                  ("edges_per_snapshot", a.edges)) if v is not None}
    if syn:
        o.setdefault("data", {})["synthetic"] = syn
    if a.snapshots is not None:
        o.setdefault("train", {})["snaps"] = int(a.snapshots)
    return o


def _scores(task: str, preds: list, targets: list | None) -> dict:
    if not targets:
        return {"samples": float(len(preds))}
    n = min(len(preds), len(targets))
    p, t = preds[:n], targets[:n]
    if task == "node_classification":  # one logit per node: positive means class 1
        return {"accuracy": sum(float(x > 0.0) == float(y) for x, y in zip(p, t)) / max(n, 1)}
    mae = sum(abs(x - y) for x, y in zip(p, t)) / max(n, 1)
    rmse = math.sqrt(sum((x - y) ** 2 for x, y in zip(p, t)) / max(n, 1))
    mean_t = abs(sum(t) / max(n, 1)) or 1.0
    return {"mae": mae, "rmse": rmse, "nmae": mae / mean_t}


def main(argv=None) -> dict:
    import torch.distributed as dist

    from starry_unigraph import SchedulerSession
    from starry_unigraph.distributed import finalize_distributed, initialize_distributed

    a = _args(argv)
    session = SchedulerSession.from_config(a.config, overrides=_overrides(a) or None)
    cfg = session.ctx.config
    if session.graph_mode != "dtdg":
        raise SystemExit(f"{a.config}: model family {cfg['model']['family']!r} is not a DTDG model")
    if a.artifact_root:
        session.ctx.artifact_root = Path(a.artifact_root).expanduser().resolve()
    rank = session.ctx.dist.rank
    log = (lambda msg: print(msg, flush=True)) if rank == 0 else (lambda msg: None)
    multi = int(os.environ.get("WORLD_SIZE", "1")) > 1
    if multi:
        initialize_distributed(session.ctx.dist)
    result: dict = {}
    try:
        if a.mode in ("prepare", "all"):
            t0 = time.perf_counter()
            if rank == 0:  # writes every rank's partition file
                session.prepare_data()
            if multi:
                dist.barrier()
            log(f"[prepare] {session.ctx.artifact_root} ({time.perf_counter() - t0:.1f}s)")
        if a.mode == "prepare":
            return result
        session.build_runtime()
        ckpt = Path(cfg["runtime"]["checkpoint"]).expanduser()
        if a.mode in ("train", "all"):
            best = math.inf
            for _ in range(int(cfg["train"]["epochs"])):
                tr = session.run_epoch("train")
                va = session.run_epoch("val")
                log(f"epoch {session.current_epoch:3d} | train loss {tr['global_loss']:.5f} "
                    f"{tr['local_steps'] / max(tr['elapsed_s'], 1e-9):.1f} snapshots/s | val loss {va['global_loss']:.5f}")
                if va["global_loss"] < best:
                    best = va["global_loss"]
                    ckpt.parent.mkdir(parents=True, exist_ok=True)
                    session.save_checkpoint(ckpt)  # rank 0 writes; parameters are identical on every rank
                result = {"train_loss": tr["global_loss"], "val_loss": va["global_loss"], "best_val_loss": best}
            log(f"[train] best val loss {best:.5f}, checkpoint {ckpt}")
        if a.mode in ("test", "all"):
            if multi:
                dist.barrier()  # rank 0's checkpoint is complete
            if ckpt.exists():
                session.load_checkpoint(ckpt)
            out = session.predict("test")
            result["test"] = _scores(cfg["model"]["task"], out.predictions, out.targets)
            log(f"[test] rank 0 partition: " + "  ".join(f"{k}={v:.5f}" for k, v in result["test"].items()))
        return result
    finally:
        if multi:
            finalize_distributed(session.ctx.dist)


if __name__ == "__main__":
    main()
