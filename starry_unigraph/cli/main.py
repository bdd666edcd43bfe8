"""Subcommand CLI (reference interface: cli/main.py:10-43):

    starry-unigraph --config CFG prepare
    starry-unigraph --config CFG train
    starry-unigraph --config CFG predict [--split S]
    starry-unigraph --config CFG resume --checkpoint PATH

Each subcommand is one entry of ``COMMANDS``: its extra arguments and the action
run on a ready session. The process group (torchrun runs) is created before the
action and torn down after it, whatever the outcome. Rank 0 prints a one-line
JSON summary of what ran.
"""
from __future__ import annotations

import argparse
import json
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any, Callable

from starry_unigraph import SchedulerSession
from starry_unigraph.distributed import finalize_distributed, initialize_distributed


def _prepare(session: SchedulerSession, args: argparse.Namespace) -> dict[str, Any]:
    """Rank 0 writes the artifacts (they do not depend on the rank); the others wait."""
    import torch.distributed as dist

    if session.ctx.dist.rank == 0:
        session.prepare_data()
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    return {"artifacts": str(session.ctx.artifact_root)}


def _train(session: SchedulerSession, args: argparse.Namespace) -> dict[str, Any]:
    out = session.run_task()
    return {"epochs": out["epochs"], "train_s": out["train_total_s"]}


def _predict(session: SchedulerSession, args: argparse.Namespace) -> dict[str, Any]:
    session.build_runtime()
    result = session.predict(split=args.split)
    return {"split": args.split, "predictions": len(result.predictions)}


def _resume(session: SchedulerSession, args: argparse.Namespace) -> dict[str, Any]:
    session.load_checkpoint(args.checkpoint)
    out = session.run_task()
    return {"checkpoint": args.checkpoint, "epochs": out["epochs"]}


@dataclass
class Command:
    action: Callable[[SchedulerSession, argparse.Namespace], dict[str, Any]]
    options: list[tuple[str, dict[str, Any]]] = field(default_factory=list)


COMMANDS: dict[str, Command] = {
    "prepare": Command(_prepare),
    "train": Command(_train),
    "predict": Command(_predict, [("--split", {"default": "test"})]),
    "resume": Command(_resume, [("--checkpoint", {"required": True})]),
}


def build_parser() -> argparse.ArgumentParser:
    parser = argparse.ArgumentParser(prog="starry-unigraph")
    parser.add_argument("--config", required=True)
    commands = parser.add_subparsers(dest="command", required=True)
    for name, spec in COMMANDS.items():
        sub = commands.add_parser(name)
        for flag, kwargs in spec.options:
            sub.add_argument(flag, **kwargs)
    return parser


def main(argv: list[str] | None = None) -> int:
    args = build_parser().parse_args(argv)
    session = SchedulerSession.from_config(Path(args.config))
    ctx = initialize_distributed(session.ctx.dist)
    try:
        summary = COMMANDS[args.command].action(session, args)
    finally:
        finalize_distributed(ctx)
    if ctx.rank == 0:
        print(json.dumps({"command": args.command} | summary, default=str), flush=True)
    return 0
