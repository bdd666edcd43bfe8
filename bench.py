"""Benchmark: TGN train events/sec on N GPUs of one node.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    torchrun --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 --master-port P bench.py --gpus N ...

Workload: synthetic unipartite event stream of the config's shape (1,140,149 nodes,
7,833,140 events, Zipf(1.2) endpoints, 20% repeat interactions, sorted uniform
timestamps over [0, 1.9e8] s, 16-dim N(0,1) edge features), random-init TGN
(memory/time/embedding 100, 2 heads, 10 most-recent neighbours, 1 mailbox slot,
1 negative per positive), 600 events per rank per step (weak scaling).

Every step is a full training step (sampling, memory update, mailbox write,
attention forward/backward, link loss, gradient all-reduce for N > 1, Adam).
``value`` is device-timed (CUDA events, W untimed warm-up steps, barrier +
synchronize on both sides, max over ranks); ``e2e`` times the public
``train_step`` API including the host->device copy of each batch from pinned
memory and the device->host read of the loss, metrics and predictions.
Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
METRIC = "TGN train events/sec & MPNN-LSTM snapshots/sec, 1/2/4/8 B200, max over ranks"
MODEL_NAME = "TGN (1-layer temporal attention, 2 heads), CTDG online + async_sync"
JODIE_NAME = "JODIE (tanh-RNN memory updater, time-projection embedding), CTDG online"


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--events", type=int, default=None,
                   help="stream length (tgn config: 7,833,140; jodie config: 200,000,000)")
    p.add_argument("--batch", type=int, default=None, help="events per rank per step (tgn: 600, jodie: 4000)")
    p.add_argument("--workload", default="tgn", choices=["tgn", "jodie", "mpnn_lstm", "tgcn", "evolvegcn"],
                   help="tgn: TGN train events/sec (default, config 3); jodie: JODIE train events/sec (config 4); "
                        "mpnn_lstm: MPNN-LSTM train snapshots/sec (config 2); tgcn / evolvegcn: config 5")
    p.add_argument("--snapshots", type=int, default=None, help="DTDG: snapshots generated (mpnn_lstm: 128, tgcn/evolvegcn: 32)")
    p.add_argument("--nodes", type=int, default=None, help="DTDG: nodes (mpnn_lstm: 200,000; tgcn/evolvegcn: 2,000,000)")
    p.add_argument("--edges", type=int, default=None,
                   help="DTDG: edges per snapshot (mpnn_lstm: 2,000,000; tgcn/evolvegcn: 20,000,000)")
    p.add_argument("--trace", action="store_true",
                   help="tgn/jodie: after the timed region, print a per-op device-time table of one eager step")
    return p.parse_args()


class ClockSampler:
    """Samples SM clock and throttle reasons of this process's GPU through NVML."""

    def __init__(self, device_index: int):
        self.samples: list[tuple[int, int]] = []
        self.reasons: set[str] = set()
        self.max_mhz = None
        self._stop = threading.Event()
        self._h = None
        try:
            import pynvml
            import torch

            pynvml.nvmlInit()
            props = torch.cuda.get_device_properties(device_index)
            bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
            self._h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
            self._nv = pynvml
        except Exception:
            self._h = None

    def _run(self):
        nv = self._nv
        names = {
            "hw_slowdown": getattr(nv, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(nv, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "sw_power_cap": getattr(nv, "nvmlClocksEventReasonSwPowerCap", 0x4),
        }
        while not self._stop.is_set():
            try:
                mhz = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, mask))
                for n, bit in names.items():
                    if mask & bit:
                        self.reasons.add(n)
            except Exception:
                pass
            time.sleep(0.05)

    def __enter__(self):
        if self._h is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._h is not None:
            self._t.join(timeout=2)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        return {"sm_mhz": statistics.median(s[0] for s in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons)}


def _reference_arm(args):
    """Run the unmodified reference from baseline/_ref through its own API."""
    ref = ROOT / "baseline" / "_ref"
    reason = None
    if not (ref / "starry_unigraph").exists():
        reason = "reference not installed under baseline/_ref"
    else:
        try:
            import dgl  # noqa: F401
        except Exception:
            reason = ("reference requires DGL (its package import chain imports dgl), which is not "
                      "installed and cannot be installed offline on this image")
    if reason is None:
        reason = "reference CTDG benchmark driver not wired"
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)
    return 0


DTDG_WORKLOADS = {
    # name: (family, task, hidden, window, preset, snapshots, nodes, edges, metric, config description)
    "mpnn_lstm": ("mpnn_lstm", "snapshot_node_regression", 64, 8, "mpnn_lstm_large", 128, 200_000, 2_000_000,
                  "MPNN-LSTM train snapshots/sec", "MPNN-LSTM (2 MPNN + 2 LSTM, hidden 64), flare_native, MSE"),
    "tgcn": ("tgcn", "node_classification", 128, 4, "egcn_large", 32, 2_000_000, 20_000_000,
             "T-GCN train snapshots/sec", "T-GCN (2 GCN layers, hidden 128, GRU-style gates), binary labels"),
    "evolvegcn": ("evolvegcn", "node_classification", 128, 4, "egcn_large", 32, 2_000_000, 20_000_000,
                  "EvolveGCN-O train snapshots/sec", "EvolveGCN-O (GCN weights evolved by a matrix GRU), binary labels"),
}


def _mpnn_main(args):
    """MPNN-LSTM: 200,000 nodes, 128 Chung-Lu snapshots of ~2M edges with 30% churn,
    64-dim features, window 8, two MPNN layers + two LSTMs of hidden 64, MSE. Nodes are partitioned over the
    ranks (strong scaling: the same graph on every N). One step = one training window ending at the next
    snapshot, so snapshots/sec = steps/sec."""
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    from starry_unigraph import SchedulerSession
    from starry_unigraph.backends.dtdg.runtime.training import run_flare_train_step
    from starry_unigraph.ops import check_status

    fam, task, hidden, window, preset, d_snaps, d_nodes, d_edges, metric_name, model_desc = DTDG_WORKLOADS[args.workload]
    snaps = args.snapshots or d_snaps
    nodes = args.nodes or d_nodes
    edges = args.edges or d_edges
    full = (snaps, nodes, edges) == (d_snaps, d_nodes, d_edges)

    def cfg(resident):
        return {
            "model": {"name": fam, "family": fam, "task": task, "hidden_dim": hidden, "window": {"size": window}},
            "data": {"root": "./data", "name": f"{fam}_large", "format": "synthetic",
                     "synthetic": {"preset": preset, "num_snapshots": snaps, "num_nodes": nodes,
                                   "edges_per_snapshot": edges}},
            "train": {"epochs": 1, "snaps": snaps, "lr": 1e-3},
            "runtime": {"device": "cuda"},
            "dtdg": {"window_from_size": True, "chunk_order": None, "chunk_decay": None, "resident": resident},
            "dist": {"backend": "nccl", "timeout_s": 1800},
        }

    session = SchedulerSession.from_config(cfg(True))
    # one artifact set for all ranks (written by rank 0): every partition file holds its
    # snapshots' features, so per-rank copies would multiply the disk footprint by N
    session.ctx.artifact_root = Path(os.environ.get("TMPDIR", "/tmp")) / f"su_{fam}_w{world}"
    if world > 1:
        from starry_unigraph.distributed import initialize_distributed

        initialize_distributed(session.ctx.dist)
    t_prep = time.perf_counter()
    if rank == 0:
        session.prepare_data()
    if world > 1:
        dist.barrier()
    session.build_runtime()
    prep_s = time.perf_counter() - t_prep
    core, rt = session.snapshot_core, session.runtime
    need = args.warmup + 2 * args.steps
    blob_list = list(core.iter_train(max_steps=need))
    if len(blob_list) < need:  # the train split holds ~70% of the snapshots
        args.steps = (len(blob_list) - args.warmup) // 2
        if args.steps <= 0:
            raise SystemExit(f"train split has only {len(blob_list)} windows")
    blobs = iter(blob_list)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        run_flare_train_step(rt, next(blobs), {"meta": {}}, need_host=False)
    torch.cuda.synchronize()
    check_status()
    timed = [next(blobs) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    from starry_unigraph.ops import cuda_ext

    launches0 = cuda_ext().launch_count()  # host-side count of this library's kernel launches
    with ClockSampler(local_rank) as clocks:
        start.record()
        h0 = time.perf_counter()
        for b in timed:
            run_flare_train_step(rt, b, {"meta": {}}, need_host=False)
        host_issue_s = time.perf_counter() - h0  # host time to issue the steps (no sync inside)
        end.record()
        torch.cuda.synchronize()
    launches = cuda_ext().launch_count() - launches0
    barrier()
    dev_ms = start.elapsed_time(end)
    check_status()
    # end to end through the per-step train call with the loss read back to the host
    # every step (the partitioned snapshots are resident on the device: no per-step H2D)
    e2e_blobs = [next(blobs) for _ in range(args.steps)]
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for b in e2e_blobs:
        float(run_flare_train_step(rt, b, {"meta": {}}, need_host=False)["loss"])  # 4-byte D2H per step
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    barrier()
    stats = torch.tensor([dev_ms, e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    dev_ms, e2e_s = float(stats[0]), float(stats[1])
    value = args.steps / (dev_ms / 1000.0)
    if rank == 0:
        print(json.dumps({
            "metric": metric_name, "value": value, "unit": "snapshots/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dev_ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32+bf16-tensor-core",
            "data": "synthetic (random-init weights)",
            "config": {"model": model_desc, "global_batch": None, "seq_len": window,
                       "parallelism": f"graph-partition{world}", "nodes": nodes, "snapshots": snaps,
                       "edges_per_snapshot": edges, "window": window, "full_config_shape": full,
                       "l2": "window graphs' CSR + features exceed the 126 MB L2", "baseline_metric": METRIC},
            "clocks": clocks.summary(), "gpu_launches": launches,
            "host_issue_ms_per_step": host_issue_s * 1000.0 / args.steps,
            "e2e": {"value": args.steps / e2e_s, "unit": "snapshots/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 4, "note": "snapshots resident on the device (dtdg.resident); "
                    "the loss is read back every step"},
            "prep_s": prep_s}), flush=True)
    if world > 1:
        from starry_unigraph.distributed import finalize_distributed

        finalize_distributed(session.ctx.dist)
    return 0


def main():
    args = _args()
    if args.impl == "reference":
        return _reference_arm(args)
    if args.workload in DTDG_WORKLOADS:
        return _mpnn_main(args)
    jodie = args.workload == "jodie"
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    from starry_unigraph import SchedulerSession
    from starry_unigraph.ops import check_status

    if args.events is None:
        args.events = 200_000_000 if jodie else 7833140
    if args.batch is None:
        args.batch = 4000 if jodie else 600
    fam, hidden, preset = ("jodie", 172, "jodie_large") if jodie else ("tgn", 100, "tgn_large")
    cfg = {
        "model": {"name": fam, "family": fam, "task": "temporal_link_prediction", "hidden_dim": hidden,
                  "memory": {"type": "rnn" if jodie else "gru"}},
        "data": {"root": "./data", "name": preset, "format": "synthetic",
                 "synthetic": {"preset": preset, "num_events": args.events, "seed": 0}},
        "train": {"epochs": 1, "batch_size": args.batch, "lr": 1e-4},
        "runtime": {"device": "cuda", "cuda_graphs": True},
        "ctdg": {"mailbox_slots": 1, "dim_time": 100, "num_head": 2, "dropout": 0.1, "att_dropout": 0.1,
                 "async_sync": True},
        "sampling": {"neighbor_limit": [10], "strategy": "recent", "history": 1},
        "graph": {"partition": "round_robin"},
        "dist": {"backend": "nccl", "timeout_s": 300},
    }
    session = SchedulerSession.from_config(cfg)
    session.ctx.artifact_root = Path(os.environ.get("TMPDIR", "/tmp")) / f"su_bench_w{world}_r{rank}"
    if world > 1:
        from starry_unigraph.distributed import initialize_distributed

        initialize_distributed(session.ctx.dist)
    t_prep = time.perf_counter()
    session.prepare_data()
    session.build_runtime()
    prep_s = time.perf_counter() - t_prep
    rt = session.ctdg_session.online_runtime
    eng = rt.engine
    need = args.warmup + 2 * args.steps
    batches = []
    for b in rt.iter_batches("train", args.batch):
        batches.append(b)
        if len(batches) >= need:
            break
    if len(batches) < need:
        raise SystemExit(f"stream too short: {len(batches)} batches < {need}")
    for b in batches:  # the loader hands out pinned batches (one H2D copy each)
        b.src, b.dst, b.ts, b.event_ids = (t.pin_memory() for t in (b.src, b.dst, b.ts, b.event_ids))

    def barrier():
        if world > 1:
            dist.barrier()

    # warm-up (includes CUDA-graph capture)
    for b in batches[: args.warmup]:
        rt._engine_step(b, "train", True, want_outputs=False)
    torch.cuda.synchronize()
    check_status()

    # ---- device-timed region
    timed = batches[args.warmup: args.warmup + args.steps]
    events = sum(b.size for b in timed)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clocks:
        start.record()
        for b in timed:
            rt._engine_step(b, "train", True, want_outputs=False)
        end.record()
        torch.cuda.synchronize()
    barrier()
    dev_ms = start.elapsed_time(end)
    check_status()

    # ---- end-to-end through the public per-step API (H2D of inputs, D2H of loss/metrics/predictions)
    e2e_batches = batches[args.warmup + args.steps: args.warmup + 2 * args.steps]
    e2e_events = sum(b.size for b in e2e_batches)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    results = session.ctdg_session.train_batches(e2e_batches)
    last = results[-1] if results else None
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    barrier()

    if args.trace and hasattr(eng, "trace_step"):
        b = e2e_batches[-1] if e2e_batches else timed[-1]
        eng.load_batch(b.src, b.dst, b.ts, b.event_ids)
        rows = eng.trace_step("train", True)
        if rank == 0:
            print(f"# per-op device time, one eager step (rank 0): {sum(t for _, t in rows):.3f} ms summed",
                  file=sys.stderr)
            for name, t in rows:
                print(f"#   {t * 1000:8.1f} us  {name}", file=sys.stderr)
    stats = torch.tensor([dev_ms, e2e_s, float(events), float(e2e_events)], dtype=torch.float64, device="cuda")
    if world > 1:
        mx = stats[:2].clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = stats[2:].clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        stats = torch.cat([mx, sm])
    dev_ms, e2e_s, events_all, e2e_events_all = stats.tolist()
    value = events_all / (dev_ms / 1000.0)
    e2e = e2e_events_all / e2e_s
    per_step_launches = eng.launches_per_step(train=True) if hasattr(eng, "launches_per_step") else None
    if rank == 0:
        bpe = 8 + 8 + 4 + 8  # src, dst, ts, eid per event
        line = {
            "metric": "JODIE train events/sec" if jodie else "TGN train events/sec",
            "value": value,
            "unit": "events/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": dev_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (random-init weights)",
            "config": {"model": JODIE_NAME if jodie else MODEL_NAME, "global_batch": args.batch * world,
                       "seq_len": None, "parallelism": f"dp{world}+memory-partition", "events": args.events,
                       "nodes": 11_000_000 if jodie else 1140149, "fanout": None if jodie else 10,
                       "mailbox_slots": 1, "dims": "memory=172, edge features 32 (bf16 on the host)" if jodie
                       else "memory=time=embed=100",
                       "l2": ("working set (memory 7.6 GB, mailbox 30 GB, edge features 25 GB) > 126 MB L2" if jodie
                              else "working set (memory 456 MB, mailbox 985 MB, edge features 500 MB) > 126 MB L2"),
                       "baseline_metric": METRIC},
            "clocks": clocks.summary(),
            "e2e": {"value": e2e, "unit": "events/s", "h2d_bytes_per_step": args.batch * bpe,
                    "d2h_bytes_per_step": 16,
                    "api": "SchedulerSession.ctdg_session.train_batches (pinned inputs copied per step, per-step "
                           "loss + AP/AUC/MRR read back per step into pinned memory)"},
            "gpu_launches": (per_step_launches * args.steps) if per_step_launches else None,
            "prep_s": prep_s,
            "last_loss": last["loss"] if last else None,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        eng.reset_graphs()
        from starry_unigraph.distributed import finalize_distributed

        finalize_distributed(session.ctx.dist)
    return 0


if __name__ == "__main__":
    sys.exit(main())
