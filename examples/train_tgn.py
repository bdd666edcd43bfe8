"""Train, validate and test a CTDG model (tgn, jodie, dyrep, tgat, apan) through
``SchedulerSession``, on one process or on every GPU of one node.

    python examples/train_tgn.py --config configs/tgn_wiki.yaml
    python examples/train_tgn.py --config configs/jodie_large.yaml --events 20000000
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 8 --master-addr 127.0.0.1 \
        --master-port 29500 examples/train_tgn.py --config configs/tgn_large_nvlink.yaml

Every epoch prints (rank 0) the train loss, the validation loss with AP / AUC / MRR, and the
training throughput in events per second over all ranks. The checkpoint of the epoch with the
best validation AP is kept (``runtime.checkpoint``; with ``--exact-resume`` every rank also
writes its memory-bank rows, optimizer moments and RNG streams), and ``--mode test`` or the
last phase of ``--mode all`` scores the test split with it. ``--resume PATH`` continues from
such a checkpoint.

Reference counterparts: examples/train_tgn.py and examples/train_tgn_dist.py of the
reference, which drive its CTDG session directly.
"""
from __future__ import annotations

import argparse
import os
import sys
import time
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))


def _args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--config", default=str(Path(__file__).resolve().parents[1] / "configs" / "tgn_wiki.yaml"))
    p.add_argument("--mode", default="all", choices=["prepare", "train", "test", "all"])
    p.add_argument("--artifact-root", default=None)
    p.add_argument("--epochs", type=int, default=None)
    p.add_argument("--batch-size", type=int, default=None, dest="batch_size")
    p.add_argument("--lr", type=float, default=None)
    p.add_argument("--device", default=None, help="cpu | cuda")
    p.add_argument("--backend", default=None, help="process-group backend: nccl (GPUs) | gloo (CPU ranks)")
    p.add_argument("--events", type=int, default=None, help="synthetic streams: first N events only")
    p.add_argument("--exact-resume", action="store_true", help="checkpoints carry the full training state")
    p.add_argument("--resume", default=None, help="checkpoint to continue from")
    return p.parse_args(argv)


def _overrides(a: argparse.Namespace) -> dict:
    o: dict = {}
    for key, val in (("epochs", a.epochs), ("batch_size", a.batch_size), ("lr", a.lr)):
        if val is not None:
            o.setdefault("train", {})[key] = val
    if a.device is not None:
        o.setdefault("runtime", {})["device"] = a.device
    if a.backend is not None:
        o.setdefault("dist", {})["backend"] = a.backend
    if a.events is not None:
        o.setdefault("data", {}).setdefault("synthetic", {})["num_events"] = int(a.events)
    return o


def _world_sum(session, value: float) -> float:
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        return value
    dev = f"cuda:{session.ctx.dist.local_rank}" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t)
    return float(t)


def _fmt(metrics: dict) -> str:
    return "  ".join(f"{k}={v:.4f}" for k, v in sorted(metrics.items()))


def main(argv=None) -> dict:
    import torch.distributed as dist

    from starry_unigraph import SchedulerSession
    from starry_unigraph.distributed import finalize_distributed, initialize_distributed

    a = _args(argv)
    session = SchedulerSession.from_config(a.config, overrides=_overrides(a) or None)
    cfg = session.ctx.config
    if session.graph_mode != "ctdg":
        raise SystemExit(f"{a.config}: model family {cfg['model']['family']!r} is not a CTDG model")
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
            if rank == 0:  # one writer; the other ranks read the artifacts in build_runtime
                session.prepare_data()
            if multi:
                dist.barrier()
            log(f"[prepare] {session.ctx.artifact_root} ({time.perf_counter() - t0:.1f}s)")
        if a.mode == "prepare":
            return result
        session.build_runtime()
        ckpt = Path(cfg["runtime"]["checkpoint"]).expanduser()
        if a.resume:
            session.load_checkpoint(a.resume)
            log(f"[resume] {a.resume} at epoch {session.current_epoch}, step {session.global_step}")
        if a.mode in ("train", "all"):
            best = -1.0
            for epoch in range(int(cfg["train"]["epochs"])):
                tr = session.run_epoch("train")
                events = _world_sum(session, float(sum(o.get("meta", {}).get("batch_size", 0) for o in tr["outputs"])))
                va = session.run_epoch("val")
                ap = float(va["metrics"].get("ap", 0.0))
                log(f"epoch {session.current_epoch:3d} | train loss {tr['loss']:.5f} "
                    f"{events / max(tr['elapsed_s'], 1e-9):,.0f} events/s | val loss {va['loss']:.5f} {_fmt(va['metrics'])}")
                if ap > best:
                    best = ap
                    ckpt.parent.mkdir(parents=True, exist_ok=True)
                    session.save_checkpoint(ckpt, exact_resume=a.exact_resume)
                result = {"train_loss": tr["loss"], "val": va["metrics"], "best_val_ap": best}
            log(f"[train] best val AP {best:.4f}, checkpoint {ckpt}")
        if a.mode in ("test", "all"):
            if multi:
                dist.barrier()  # rank 0's checkpoint is complete
            if ckpt.exists():
                session.load_checkpoint(ckpt)
            te = session.evaluate("test")
            result["test"] = te["metrics"]
            log(f"[test] loss {te['loss']:.5f} {_fmt(te['metrics'])}")
        return result
    finally:
        if multi:
            finalize_distributed(session.ctx.dist)  # every epoch ended with the peers' write-backs landed


if __name__ == "__main__":
    main()
