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
    # generous: on a cold machine the first torch import of each rank can take a minute
    p.add_argument("--timeout", type=float, default=240.0)
    p.add_argument("--heartbeat", type=float, default=0.0)
    p.add_argument("--resume", action="store_true",
                   help="CTDG: train K1 + K2 steps, and K1 steps -> exact-resume checkpoint -> new session -> K2 steps")
    p.add_argument("--ctdg-json", default=None, help="JSON object merged into the config's ctdg section")
    p.add_argument("--chunk", type=int, default=0,
                   help="> 0: chunk mode with this many node clusters on a synthetic stream, then predict")
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
    if a.ctdg_json:
        cfg["ctdg"].update(json.loads(a.ctdg_json))
    if a.chunk:
        cfg["data"] = {"root": str(Path(a.out) / "data"), "name": "dist_chunk", "format": "synthetic",
                       "graph_mode": "chunk", "synthetic": {"preset": "tgn_cpu", "num_events": 2000}}
        cfg["chunk"] = {"node_clusters": a.chunk, "time_slices": 4}
        cfg["train"]["batch_size"] = 64
    s = SchedulerSession.from_config(cfg)
    # chunk mode: one artifact set (rank 0 writes it) whose partition files every rank reads
    s.ctx.artifact_root = Path(a.out) / ("art" if a.chunk else f"art_r{rank}")
    initialize_distributed(s.ctx.dist)
    if a.resume:
        _resume_check(a, cfg, s, rank)
        finalize_distributed(s.ctx.dist)
        os._exit(0)
    t0 = time.time()
    outcome = {"rank": rank, "error": None}
    try:
        if a.chunk:
            import torch.distributed as dist

            if rank == 0:
                s.prepare_data()
            dist.barrier()
        else:
            s.prepare_data()
        s.build_runtime()
        r = s.run_epoch("train")
        if a.chunk:
            outcome["local_steps"] = r["local_steps"]
            outcome["own_chunks"] = len(list(s.snapshot_core.iter_chunks("train")))
            outcome["val_steps"] = s.run_epoch("val")["local_steps"]
            # the unified engine over the same runtime walks the same lock-step units
            eng = s.build_pipeline_engine()
            outcome["engine_losses"] = len(eng.run_epoch("train", batch_size=64)["losses"])
            ckpt = Path(a.out) / "ckpt" / "chunk.pt"
            s.save_checkpoint(ckpt)
            s.load_checkpoint(ckpt)  # every rank reads the file rank 0 wrote
            outcome["predictions"] = len(s.predict("test").predictions)
        outcome["steps"] = r["steps"]
        outcome["loss"] = r["loss"]
        outcome["alphas"] = [o["meta"].get("historical_alpha") for o in r["outputs"]
                             if "historical_alpha" in o.get("meta", {})]
        if ctdg and not a.chunk:
            outcome.update(_pull_check(s))
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


def _pull_check(s):
    """Rows pulled during the epoch, and whether pulling every remote row now returns
    exactly the owners' rows (after all pushes have landed)."""
    import torch
    import torch.distributed as dist

    mem = s.ctdg_session.online_runtime.memory
    pulled = mem.pulled_rows
    mem.wait_pending_syncs()
    dist.barrier()
    if not mem.remote_fetch:
        return {"pulled": pulled}
    mem.pull_remote(s.ctx.dist, torch.arange(mem.num_nodes))
    tables = [torch.zeros_like(mem.memory) for _ in range(dist.get_world_size())]
    dist.all_gather(tables, mem.memory)
    owners_view = torch.stack(tables)[mem.owner, torch.arange(mem.num_nodes)]
    return {"pulled": pulled, "pull_exact": bool(torch.equal(owners_view, mem.memory))}


def _resume_check(a, cfg, s, rank):
    """Uninterrupted run against save / fresh session / load / continue."""
    import torch

    from starry_unigraph import SchedulerSession

    k1, k2 = 3, 4
    s.prepare_data()
    s.build_runtime()
    batches = list(s.ctdg_session.online_runtime.iter_batches("train", 8))[: k1 + k2]
    full = [float(s.ctdg_session.train_step(b)["loss"]) for b in batches]
    mem_full = s.ctdg_session.online_runtime.memory

    def fresh():
        t = SchedulerSession.from_config(cfg)
        t.ctx.artifact_root = s.ctx.artifact_root
        t.build_runtime()
        return t

    first = fresh()
    for b in batches[:k1]:
        first.ctdg_session.train_step(b)
    ckpt = Path(a.out) / "ckpt" / "resume.pt"
    first.save_checkpoint(ckpt, exact_resume=True)
    second = fresh()
    second.load_checkpoint(ckpt)
    rest = [float(second.ctdg_session.train_step(b)["loss"]) for b in batches[k1:]]
    m2 = second.ctdg_session.online_runtime.memory
    model_a = s.runtime.model.module if hasattr(s.runtime.model, "module") else s.runtime.model
    model_b = second.runtime.model.module if hasattr(second.runtime.model, "module") else second.runtime.model
    mem_full.wait_pending_syncs()
    m2.wait_pending_syncs()
    torch.save({"full": full[k1:], "resumed": rest,
                "params_full": [p.detach().clone() for p in model_a.parameters()],
                "params_resumed": [p.detach().clone() for p in model_b.parameters()],
                "memory_full": mem_full.memory.clone(), "memory_resumed": m2.memory.clone(),
                "mailbox_full": mem_full.mailbox.clone(), "mailbox_resumed": m2.mailbox.clone(),
                "rank_file": SchedulerSession.rank_state_path(ckpt, rank).exists()},
               Path(a.out) / f"resume_r{rank}.pt")


if __name__ == "__main__":
    main()
