"""Subcommand CLI (reference cli/main.py:10-43):
``starry-unigraph --config X {prepare,train,predict [--split S],resume --checkpoint P}``."""
from __future__ import annotations

import argparse
from pathlib import Path

from starry_unigraph import SchedulerSession
from starry_unigraph.distributed import finalize_distributed, initialize_distributed


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="starry-unigraph")
    p.add_argument("--config", required=True)
    sub = p.add_subparsers(dest="command", required=True)
    sub.add_parser("prepare")
    sub.add_parser("train")
    pr = sub.add_parser("predict")
    pr.add_argument("--split", default="test")
    rs = sub.add_parser("resume")
    rs.add_argument("--checkpoint", required=True)
    return p


def main(argv: list[str] | None = None) -> int:
    args = build_parser().parse_args(argv)
    session = SchedulerSession.from_config(Path(args.config))
    initialize_distributed(session.ctx.dist)
    try:
        if args.command == "prepare":
            session.prepare_data()
        elif args.command == "train":
            session.run_task()
        elif args.command == "predict":
            session.build_runtime()
            session.predict(split=args.split)
        elif args.command == "resume":
            session.load_checkpoint(args.checkpoint)
            session.run_task()
    finally:
        finalize_distributed(session.ctx.dist)
    return 0
