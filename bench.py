"""Benchmark: TGN train events/sec on N GPUs of one node, with the
MPNN-LSTM snapshots/sec of config 2 nested in the same JSON line (``mpnn_lstm``).

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
    p.add_argument("--workload", default="tgn", choices=["tgn", "jodie", "mpnn_lstm", "tgcn", "evolvegcn", "tgn_cpu"],
                   help="tgn: TGN train events/sec (default, config 3); jodie: JODIE train events/sec (config 4); "
                        "mpnn_lstm: MPNN-LSTM train snapshots/sec (config 2); tgcn / evolvegcn: config 5; "
                        "tgn_cpu: TGN train events/sec in one CPU process (config 1), host-timed")
    p.add_argument("--snapshots", type=int, default=None, help="DTDG: snapshots generated (mpnn_lstm: 128, tgcn/evolvegcn: 32)")
    p.add_argument("--nodes", type=int, default=None, help="DTDG: nodes (mpnn_lstm: 200,000; tgcn/evolvegcn: 2,000,000)")
    p.add_argument("--edges", type=int, default=None,
                   help="DTDG: edges per snapshot (mpnn_lstm: 2,000,000; tgcn/evolvegcn: 20,000,000)")
    p.add_argument("--trace", action="store_true",
                   help="tgn/jodie: after the timed region, print a per-op device-time table of one eager step")
    p.add_argument("--no-mpnn", action="store_true",
                   help="default workload: skip the nested MPNN-LSTM (config 2) measurement")
    p.add_argument("--mpnn-steps", type=int, default=40,
                   help="default workload: timed MPNN-LSTM windows (at most the train split's windows)")
    p.add_argument("--no-graphs", action="store_true", help="DTDG: eager steps instead of CUDA-graph replays")
    p.add_argument("--dtdg-precision", default="bf16", choices=["tf32", "bf16"],
                   help="DTDG tensor-core operand precision (config 2 names fp32/bf16, config 5 bf16)")
    p.add_argument("--precision", default="tf32", choices=["tf32", "bf16"],
                   help="tensor-core operand precision of the headline (runtime.precision)")
    p.add_argument("--no-bf16", action="store_true", help="tgn/jodie: skip the nested bf16 measurement")
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
    """Run the unmodified reference from baseline/_ref through its own public API
    (bench_reference.py in a subprocess whose import path holds only the reference),
    on the same synthetic stream; print its JSON line, or an ``unavailable`` line."""
    import subprocess
    import tempfile

    rank = int(os.environ.get("RANK", "0"))

    def unavailable(reason: str) -> int:
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": reason}), flush=True)
        return 0

    ref = ROOT / "baseline" / "_ref"
    if not (ref / "starry_unigraph").exists():
        return unavailable("reference not installed under baseline/_ref")
    env = dict(os.environ)
    env["PYTHONPATH"] = str(ref)
    scratch = Path(tempfile.mkdtemp(prefix=f"su_ref_r{rank}_"))
    probe = subprocess.run([sys.executable, "-c", "import dgl, starry_unigraph.session"], cwd=scratch, env=env,
                           capture_output=True, text=True)
    if probe.returncode != 0:
        last = (probe.stderr.strip().splitlines() or ["import failed"])[-1]
        return unavailable("reference requires DGL (its package import chain imports dgl), which is not installed "
                           f"and has no offline wheel on this image ({last})")
    if args.workload != "tgn":
        return unavailable(f"reference arm is wired for the headline TGN workload, not {args.workload}")
    # the workload in the reference's CSV format (data/raw_temporal.py): edges.csv + edge_features.pt
    sys.path.insert(0, str(ROOT))
    import pandas as pd
    import torch

    from starry_unigraph.data.synthetic import ctdg_preset

    stream = ctdg_preset("tgn_large", num_events=args.events or 7833140, seed=0)
    ds = scratch / "data" / "tgn_large"
    ds.mkdir(parents=True, exist_ok=True)
    pd.DataFrame({"src": stream["src"].numpy(), "dst": stream["dst"].numpy(),
                  "time": stream["ts"].numpy()}).to_csv(ds / "edges.csv", index=False)
    torch.save(stream["edge_feat"].float(), ds / "edge_features.pt")
    driver = ROOT / "bench_reference.py"
    cmd = [sys.executable, "-c", f"import runpy; runpy.run_path({str(driver)!r}, run_name='__main__')",
           "--data", str(scratch / "data"), "--name", "tgn_large", "--steps", str(args.steps),
           "--warmup", str(args.warmup), "--batch", str(args.batch or 600)]
    run = subprocess.run(cmd, cwd=scratch, env=env, capture_output=True, text=True)
    lines = [ln for ln in run.stdout.splitlines() if ln.startswith("{")]
    if run.returncode != 0 or (rank == 0 and not lines):
        last = (run.stderr.strip().splitlines() or ["no output"])[-1]
        return unavailable(f"reference run failed: {last}")
    if rank == 0:
        print(lines[-1], flush=True)
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


def _dtdg_run(args, workload: str, steps: int, warmup: int) -> dict:
    """DTDG snapshot throughput on the workload's BASELINE.json shape. mpnn_lstm (config 2): 200,000 nodes,
    128 Chung-Lu snapshots of ~2M edges with 30% churn, 64-dim features, window 8, two MPNN layers + two LSTMs
    of hidden 64, MSE. Nodes are partitioned over the ranks (strong scaling: the same graph on every N). One
    step = one training window ending at the next snapshot, so snapshots/sec = steps/sec.

    Steps run as CUDA graphs of the whole window step (forward, backward, Adam): the timed windows are
    captured in an untimed pass after the warm-up, then the timed pass replays them (full work every replay,
    parameters change every step); the end-to-end pass replays them once more through the public per-step
    call with the loss read back each step. The process group must already be initialised for N > 1."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    from starry_unigraph import SchedulerSession
    from starry_unigraph.backends.dtdg.runtime.training import run_flare_train_step
    from starry_unigraph.ops import check_status, cuda_ext

    fam, task, hidden, window, preset, d_snaps, d_nodes, d_edges, metric_name, model_desc = DTDG_WORKLOADS[workload]
    snaps = args.snapshots or d_snaps
    nodes = args.nodes or d_nodes
    edges = args.edges or d_edges
    full = (snaps, nodes, edges) == (d_snaps, d_nodes, d_edges)
    cfg = {
        "model": {"name": fam, "family": fam, "task": task, "hidden_dim": hidden, "window": {"size": window}},
        "data": {"root": "./data", "name": f"{fam}_large", "format": "synthetic",
                 "synthetic": {"preset": preset, "num_snapshots": snaps, "num_nodes": nodes,
                               "edges_per_snapshot": edges}},
        "train": {"epochs": 1, "snaps": snaps, "lr": 1e-3},
        "runtime": {"device": "cuda", "cuda_graphs": not args.no_graphs, "precision": args.dtdg_precision},
        "dtdg": {"window_from_size": True, "chunk_order": None, "chunk_decay": None, "resident": True},
        "dist": {"backend": "nccl", "timeout_s": 1800},
    }
    session = SchedulerSession.from_config(cfg)
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
    graphs = rt.state.get("step_graphs")
    blob_list = list(core.iter_train())  # frozen windows of the train split
    steps = max(1, min(steps, len(blob_list) - warmup))
    warm, timed = blob_list[:warmup], blob_list[warmup:warmup + steps]

    def barrier():
        if world > 1:
            dist.barrier()

    barrier()  # ranks enter the first step (and its device-side halo barriers) together
    torch.cuda.synchronize()
    for b in warm:
        run_flare_train_step(rt, b, {"meta": {}}, need_host=False)
    if graphs is not None:
        for b in timed:  # capture pass (untimed): one graph per timed window
            run_flare_train_step(rt, b, {"meta": {}}, need_host=False)
    torch.cuda.synchronize()
    check_status()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
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
    if graphs is not None:
        # replays issue no host-side launches; the count comes from the captured (eager) steps
        launches = int(graphs.launches_per_step * steps)
    barrier()
    dev_ms = start.elapsed_time(end)
    check_status()
    # end to end through the per-step train call with the loss read back to the host every step
    # (the partitioned snapshots are resident on the device: no per-step H2D)
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    last_loss = None
    for b in timed:
        last_loss = float(run_flare_train_step(rt, b, {"meta": {}}, need_host=False)["loss"])  # 4-byte D2H
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    barrier()
    # this rank's own device time and work (edges of every window graph it aggregated, its rows)
    own_edges = sum(int(st.graph.edge_src.numel()) for b in timed for st in b.steps)
    own_rows = int(timed[0].steps[-1].graph.num_dst_nodes) if timed and timed[0].steps else 0
    mine = torch.tensor([dev_ms, float(own_edges), float(own_rows)], dtype=torch.float64, device="cuda")
    per_rank = [mine]
    if world > 1:
        per_rank = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(per_rank, mine)
    stats = torch.tensor([dev_ms, e2e_s], dtype=torch.float64, device="cuda")
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    dev_ms, e2e_s = float(stats[0]), float(stats[1])
    out = {
        "metric": metric_name, "value": steps / (dev_ms / 1000.0), "unit": "snapshots/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": dev_ms / steps, "higher_is_better": True,
        "scaling": "strong", "dtype": "tf32" if rt.state.get("precision_tf32") else "bf16",
        "dtype_detail": ("tf32" if rt.state.get("precision_tf32") else "bf16") +
        " tensor-core operands, fp32 storage and accumulation (SpMM, LSTM gates and Adam in fp32)",
        "data": "synthetic (random-init weights)",
        "config": {"model": model_desc, "global_batch": None, "seq_len": window,
                   "parallelism": f"graph-partition{world}", "nodes": nodes, "snapshots": snaps,
                   "edges_per_snapshot": edges, "window": window, "full_config_shape": full,
                   "cuda_graphs": graphs is not None,
                   "capture_pass": ("each timed window captured once in an untimed pass before timing"
                                    if graphs is not None else None),
                   "l2": "window graphs' CSR + features exceed the 126 MB L2"},
        "clocks": clocks.summary(), "gpu_launches": launches,
        "host_issue_ms_per_step": host_issue_s * 1000.0 / steps,
        "e2e": {"value": steps / e2e_s, "unit": "snapshots/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4,
                "note": "snapshots resident on the device (dtdg.resident); the loss is read back every step"},
        "prep_s": prep_s, "last_loss": last_loss,
        # per rank: device ms per step, aggregated edges per step (all window graphs), owned rows
        "per_rank": [{"ms_per_step": round(float(t[0]) / steps, 3), "edges_per_step": int(float(t[1]) / steps),
                      "rows": int(t[2])} for t in per_rank],
    }
    if world > 1:
        out["consistency"] = _replicas_equal(rt.optimizer.flat.data if hasattr(rt.optimizer, "flat") else
                                             torch.cat([p.detach().view(-1) for p in rt.model.parameters()]))
    if graphs is not None:
        graphs.reset()
    return out


def _replicas_equal(flat) -> dict:
    """Cross-rank check: every rank's parameter buffer is bit-identical (float64 sum and max abs
    difference against rank 0's copy)."""
    import torch
    import torch.distributed as dist

    ref = flat.detach().clone()
    dist.broadcast(ref, src=0)
    diff = torch.tensor([float((flat.detach() - ref).abs().max())], dtype=torch.float64, device=flat.device)
    dist.all_reduce(diff, op=dist.ReduceOp.MAX)
    return {"params_max_abs_diff_vs_rank0": float(diff), "params_equal": float(diff) == 0.0}


def _mpnn_main(args):
    import torch

    sys.path.insert(0, str(ROOT))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    out = _dtdg_run(args, args.workload, args.steps, args.warmup)
    out["vs_baseline"] = None
    out["config"]["baseline_metric"] = METRIC
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps(out), flush=True)
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
    return 0


def _ctdg_run(args, precision: str = "tf32") -> dict:
    """TGN (config 3) or JODIE (config 4) events/sec with the given tensor-core operand precision
    (runtime.precision); the process group must be initialised for N > 1."""
    jodie = args.workload == "jodie"
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
        "runtime": {"device": "cuda", "cuda_graphs": True, "precision": precision},
        "ctdg": {"mailbox_slots": 1, "dim_time": 100, "num_head": 2, "dropout": 0.1, "att_dropout": 0.1,
                 "async_sync": True},
        "sampling": {"neighbor_limit": [10], "strategy": "recent", "history": 1},
        "graph": {"partition": "round_robin"},
        "dist": {"backend": "nccl", "timeout_s": 1800},
    }
    session = SchedulerSession.from_config(cfg)
    session.ctx.artifact_root = Path(os.environ.get("TMPDIR", "/tmp")) / f"su_bench_{precision}_w{world}_r{rank}"
    if world > 1:
        from starry_unigraph.distributed import initialize_distributed

        initialize_distributed(session.ctx.dist)  # the process group exists: records it in the context
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

    # warm-up (includes CUDA-graph capture); ranks enter the first step together
    barrier()
    torch.cuda.synchronize()
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

    phases = None
    if args.trace and hasattr(eng, "trace_step"):
        # per-op device times of eager steps (after the timed region), summed into the phases of
        # the multi-GPU step; the wait phase absorbs the peers' lateness (load imbalance)
        phase_of = {"tgn_peer_wait_claim": "end_wait_and_claims", "peer_barrier": "barrier_grads_complete",
                    "tgn_peer_push": "writeback_push_side_stream", "peer_rs_adam_ag": "reduce_scatter_adam_allgather",
                    "peer_signal": "end_signal"}
        names = ["compute"] + list(phase_of.values())
        acc = dict.fromkeys(names, 0.0)
        src = (e2e_batches or timed)[-5:]
        rows = []
        for b in src:
            eng.load_batch(b.src, b.dst, b.ts, b.event_ids)
            rows = eng.trace_step("train", True)
            for name, t in rows:
                acc[phase_of.get(name, "compute")] += t
        mine_p = torch.tensor([acc[n] / max(1, len(src)) for n in names], dtype=torch.float64, device="cuda")
        gathered = [mine_p]
        if world > 1:
            gathered = [torch.empty_like(mine_p) for _ in range(world)]
            dist.all_gather(gathered, mine_p)
        phases = {n: [round(float(g[i]), 4) for g in gathered] for i, n in enumerate(names)}
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
        "dtype": "tf32" if precision == "tf32" else "bf16",
        "dtype_detail": (f"{precision} tensor-core operands (kind::{'tf32' if precision == 'tf32' else 'f16'}), "
                         "fp32 storage and accumulation"),
        "data": "synthetic (random-init weights)",
        "config": {"model": JODIE_NAME if jodie else MODEL_NAME, "global_batch": args.batch * world,
                   "seq_len": None, "parallelism": f"dp{world}+memory-partition", "events": args.events,
                   "nodes": 11_000_000 if jodie else 1140149, "fanout": None if jodie else 10,
                   "mailbox_slots": 1, "dims": "memory=172, edge features 32 (bf16 on the host)" if jodie
                   else "memory=time=embed=100",
                   "event_assignment": rt.dataset.assignment if world > 1 else None,
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
    eng.drain()
    if world > 1:
        cons = _replicas_equal(eng.flat.data)
        mem = rt.memory
        stray = ((mem.memory_ts >= 0) & (mem.owner != rank)).sum().to(torch.float64).view(1)
        dist.all_reduce(stray)
        cons["rows_written_on_non_owners"] = int(stray)
        cons["peer_path"] = eng.peer is not None
        line["consistency"] = cons
    if phases is not None:
        # --trace: device ms per step and phase (eager steps, CUDA events around every op), one value per rank
        line["phases_ms_per_step"] = phases
    eng.reset_graphs()
    return line


def _tgn_cpu_run(args) -> int:
    """TGN (1-layer attention, 2 heads, memory / time / embedding 100,
    GRU updater, one mailbox slot, 10 recent neighbours) in one CPU process, fp32, on the
    9,227-node / 157,474-event Zipf(1.1) stream with 172-dim edge features, batch 200, one
    negative per event, 70/15/15 split. Steps go through the public per-batch API
    (``SchedulerSession.ctdg_session.train_step``) and are timed with the host clock (no GPU
    involved): W untimed steps, then K timed ones."""
    import tempfile

    import torch

    sys.path.insert(0, str(ROOT))
    from starry_unigraph import SchedulerSession

    cfg = {"model": {"name": "tgn", "family": "tgn", "task": "temporal_link_prediction", "hidden_dim": 100},
           "data": {"root": "./data", "name": "tgn_cpu", "format": "synthetic", "synthetic": {"preset": "tgn_cpu"}},
           "train": {"epochs": 1, "batch_size": args.batch or 200, "lr": 1e-4},
           "runtime": {"device": "cpu"},
           "ctdg": {"mailbox_slots": 1, "dim_time": 100, "num_head": 2, "dropout": 0.1, "att_dropout": 0.1},
           "sampling": {"neighbor_limit": [10], "strategy": "recent", "history": 1}}
    session = SchedulerSession.from_config(cfg)
    session.ctx.artifact_root = Path(tempfile.mkdtemp(prefix="su_tgn_cpu_"))
    session.prepare_data()
    session.build_runtime()
    rt = session.ctdg_session.online_runtime
    batches = []
    for b in rt.iter_batches("train", args.batch or 200):
        batches.append(b)
        if len(batches) >= args.warmup + args.steps:
            break
    for b in batches[: args.warmup]:
        session.ctdg_session.train_step(b)
    timed = batches[args.warmup:]
    events = sum(int(b.size) for b in timed)
    t0 = time.perf_counter()
    for b in timed:
        session.ctdg_session.train_step(b)
    wall = time.perf_counter() - t0
    print(json.dumps({"metric": "TGN train events/sec (CPU, single process)", "value": events / wall,
                      "unit": "events/s", "n_gpus": 0, "device": "cpu", "threads": torch.get_num_threads(),
                      "steps": len(timed), "warmup": args.warmup, "ms_per_step": wall * 1000.0 / max(1, len(timed)),
                      "higher_is_better": True, "scaling": "none", "vs_baseline": None, "dtype": "fp32",
                      "data": "synthetic (random-init weights)", "timing": "host clock (perf_counter)",
                      "config": {"model": "TGN (1-layer temporal attention, 2 heads), CPU", "global_batch": args.batch or 200,
                                 "events": 157474, "nodes": 9227, "edge_dim": 172, "fanout": 10}}), flush=True)
    return 0


def main():
    args = _args()
    if args.impl == "reference":
        return _reference_arm(args)
    if args.workload == "tgn_cpu":
        return _tgn_cpu_run(args)
    import torch

    if not torch.cuda.is_available():
        print(f"bench.py: the {args.workload} workload runs on CUDA devices and none is visible here "
              "(--workload tgn_cpu measures the CPU configuration)", file=sys.stderr)
        return 2
    if args.workload in DTDG_WORKLOADS:
        return _mpnn_main(args)
    sys.path.insert(0, str(ROOT))
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=1800),
                                device_id=torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0"))))
    line = _ctdg_run(args, args.precision)
    if args.precision == "tf32" and not args.no_bf16:
        # the same step with bf16 tensor-core operands, reported separately (device-timed)
        fast = _ctdg_run(args, "bf16")
        line["bf16"] = {k: fast[k] for k in ("metric", "value", "unit", "ms_per_step", "dtype", "dtype_detail",
                                              "clocks")} | {"e2e": fast["e2e"]["value"]}
    if args.workload == "tgn" and not args.no_mpnn:
        # BASELINE.json's headline pairs TGN events/sec with MPNN-LSTM snapshots/sec (config 2): measured in
        # the same run, reported nested, with its own device timing, clocks and end-to-end rate
        line["mpnn_lstm"] = _dtdg_run(args, "mpnn_lstm", args.mpnn_steps, max(3, args.warmup))
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
