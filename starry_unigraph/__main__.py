"""Command line entry point (reference __main__.py:1-272).

    python -m starry_unigraph --config CONFIG [--phase prepare|train|predict|all]
                              [--artifact-root PATH] [--epochs N] [--lr F] [--batch-size N] [--device DEV]

The graph mode comes from ``data.graph_mode`` or ``model.family``. ``train``
runs train + validation every epoch and writes the checkpoint (rank 0);
``predict`` loads the checkpoint when present and prints MAE / RMSE / NMAE on
rank 0. Use torchrun for several GPUs.
"""
from __future__ import annotations

import argparse
import math
import os
import time
from pathlib import Path


def _rank() -> int:
    return int(os.environ.get("RANK", "0"))


def _log(msg: str) -> None:
    if _rank() == 0:
        print(f"[rank {_rank()}] {msg}", flush=True)


def _parse_args(argv=None) -> argparse.Namespace:
    p = argparse.ArgumentParser(prog="python -m starry_unigraph", description="starry_unigraph entry point",
                                formatter_class=argparse.RawDescriptionHelpFormatter, epilog=__doc__)
    p.add_argument("--config", required=True, metavar="PATH")
    p.add_argument("--phase", default="all", choices=["prepare", "train", "predict", "all"])
    p.add_argument("--artifact-root", default=None, metavar="PATH")
    p.add_argument("--epochs", type=int, default=None)
    p.add_argument("--lr", type=float, default=None)
    p.add_argument("--batch-size", type=int, default=None, dest="batch_size")
    p.add_argument("--device", default=None)
    return p.parse_args(argv)


def _build_session(args: argparse.Namespace):
    from starry_unigraph.config.schema import load_config, validate_config
    from starry_unigraph.distributed import apply_distributed_env, build_distributed_context
    from starry_unigraph.registry import ModelRegistry, TaskRegistry
    from starry_unigraph.session import SchedulerSession
    from starry_unigraph.types import SessionContext

    overrides: dict = {}
    if args.epochs is not None:
        overrides.setdefault("train", {})["epochs"] = args.epochs
    if args.lr is not None:
        overrides.setdefault("train", {})["lr"] = args.lr
    if args.batch_size is not None:
        overrides.setdefault("train", {})["batch_size"] = args.batch_size
    if args.device is not None:
        overrides.setdefault("runtime", {})["device"] = args.device
    config = apply_distributed_env(load_config(args.config, overrides=overrides or None))
    warnings = validate_config(config)
    for w in warnings:
        _log(f"[warn] {w}")
    spec = ModelRegistry.resolve(model_name=config["model"]["name"], family=config["model"]["family"])
    task_cls = TaskRegistry.resolve(config["model"]["task"])
    # artifact root: CLI flag > parent of the checkpoint directory > ./artifacts/<name>
    if args.artifact_root:
        root = Path(args.artifact_root).expanduser().resolve()
    else:
        ckpt = config.get("runtime", {}).get("checkpoint", "")
        root = Path(ckpt).expanduser().resolve().parent.parent if ckpt else \
            (Path.cwd() / "artifacts" / config["data"]["name"]).resolve()
    ctx = SessionContext(config=config, project_root=Path(args.config).expanduser().resolve().parent,
                         dataset_path=None, artifact_root=root, dist=build_distributed_context(config),
                         warnings=warnings)
    return SchedulerSession(session_ctx=ctx, model_spec=spec, task_adapter=task_cls())


def _run_prepare(args) -> None:
    s = _build_session(args)
    _log(f"[prepare] artifact_root = {s.ctx.artifact_root}")

    def body():
        # the artifacts do not depend on the rank: rank 0 writes them while the others wait,
        # so no rank reads a file that another is still writing
        t0 = time.perf_counter()
        if _rank() == 0:
            s.ctx.artifact_root.mkdir(parents=True, exist_ok=True)
            s.prepare_data()
        if int(os.environ.get("WORLD_SIZE", "1")) > 1:
            import torch.distributed as dist

            dist.barrier()
        _log(f"[prepare] done in {time.perf_counter() - t0:.1f}s")

    _with_dist(s, body)


def _with_dist(s, fn):
    """Run `fn` with the process group up. One group serves every phase of the run (the
    first phase creates it, later ones adopt it; ``main`` tears it down at the end):
    re-creating it between phases costs a rendezvous and can stall."""
    from starry_unigraph.distributed import initialize_distributed

    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        initialize_distributed(s.ctx.dist)
    return fn()


def _run_train(args) -> None:
    s = _build_session(args)
    _log(f"[train] artifact_root = {s.ctx.artifact_root}")

    def body():
        s.build_runtime()
        epochs = int(s.ctx.config["train"]["epochs"])
        _log(f"[train] graph_mode={s.ctx.config['data'].get('graph_mode')}  epochs={epochs}")
        for epoch in range(epochs):
            t0 = time.perf_counter()
            tr = s.run_epoch(split="train")
            t1 = time.perf_counter()
            ev = s.run_epoch(split="val")
            if _rank() == 0:
                print(f"epoch {epoch + 1:3d}/{epochs} | train_loss={tr.get('loss', float('nan')):.6f} ({t1 - t0:.2f}s)"
                      f" | val_loss={ev.get('loss', float('nan')):.6f} ({time.perf_counter() - t1:.2f}s)", flush=True)
        ckpt = Path(s.ctx.config["runtime"].get("checkpoint", "checkpoint.pt"))
        ckpt.parent.mkdir(parents=True, exist_ok=True)
        s.save_checkpoint(ckpt)
        _log(f"[train] checkpoint saved -> {ckpt}")

    _with_dist(s, body)


def _run_predict(args) -> None:
    s = _build_session(args)
    _log(f"[predict] artifact_root = {s.ctx.artifact_root}")

    def body():
        s.build_runtime()
        ckpt = Path(s.ctx.config["runtime"].get("checkpoint", "checkpoint.pt"))
        if ckpt.exists():
            s.load_checkpoint(ckpt)
            _log(f"[predict] loaded checkpoint <- {ckpt}")
        else:
            _log(f"[predict] no checkpoint at {ckpt}, using init model")
        t0 = time.perf_counter()
        result = s.predict(split="test")
        elapsed = time.perf_counter() - t0
        if _rank() == 0:
            preds, tgts = result.predictions, result.targets or []
            print(f"\n=== predict done in {elapsed:.2f}s - {len(preds)} samples ===")
            if tgts:
                n = min(len(preds), len(tgts))
                mae = sum(abs(p - t) for p, t in zip(preds[:n], tgts[:n])) / n
                rmse = math.sqrt(sum((p - t) ** 2 for p, t in zip(preds[:n], tgts[:n])) / n)
                mean_t = sum(tgts[:n]) / n or 1.0
                print(f"  MAE={mae:.6f}  RMSE={rmse:.6f}  NMAE={mae / abs(mean_t):.6f}")
            print(flush=True)

    _with_dist(s, body)


def main(argv=None) -> None:
    args = _parse_args(argv)
    _log(f"config={args.config}  phase={args.phase}")
    try:
        if args.phase in ("prepare", "all"):
            _run_prepare(args)
        if args.phase in ("train", "all"):
            _run_train(args)
        if args.phase in ("predict", "all"):
            _run_predict(args)
    finally:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
