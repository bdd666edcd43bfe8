"""Multi-rank runs on CPU (gloo) through the public session API: DTDG halo
exchange and data-parallel gradients, CTDG memory partitioning (two and four
ranks), and failure detection on the host (a rank that exits between steps)."""
import json
import math
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parents[1]
WORKER = ROOT / "tests" / "workers" / "dist_cpu_worker.py"


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _launch(out, family, extra_env=None, *args, wall=420, nproc=2):
    env = dict(os.environ)
    env.pop("CUDA_VISIBLE_DEVICES", None)
    env.update(extra_env or {})
    for attempt in range(3):  # a port picked free can be taken before the rendezvous binds it
        cmd = ["timeout", "-k", "10", str(wall), sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1", "--master-port", str(_port()), str(WORKER),
               "--family", family, "--out", str(out), *args]
        res = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=wall + 30)
        text = res.stdout + res.stderr
        if res.returncode == 0 or not any(m in text for m in ("Address already in use", "EADDRINUSE", "errno: 98")):
            return res
    return res


def _outcome(out, r):
    return json.loads((Path(out) / f"outcome_r{r}.json").read_text())


def test_dtdg_two_ranks_halo_and_gradients(tmp_path):
    res = _launch(tmp_path, "mpnn_lstm")
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    o0, o1 = _outcome(tmp_path, 0), _outcome(tmp_path, 1)
    assert o0["error"] is None and o1["error"] is None
    assert o0["steps"] == o1["steps"] > 0
    p0, p1 = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    # one all-reduced gradient buffer per step: replicas stay identical
    for a, b in zip(p0["params"], p1["params"]):
        assert torch.allclose(a, b, atol=1e-6)


def test_ctdg_two_ranks_memory_partition(tmp_path):
    res = _launch(tmp_path, "tgn")
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    o0, o1 = _outcome(tmp_path, 0), _outcome(tmp_path, 1)
    assert o0["error"] is None and o1["error"] is None
    p0, p1 = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    for a, b in zip(p0["params"], p1["params"]):
        assert torch.allclose(a, b, atol=1e-6)


@pytest.mark.parametrize("adaptive", [True, False])
def test_ctdg_historical_cache_alpha(tmp_path, adaptive):
    """Remote reads off (the reference's push path): the historical cache filters the
    pushed rows; with ada_param_enabled its alpha follows each step's sync / compute
    time within its bounds, without it alpha stays at historical_alpha."""
    over = json.dumps({"remote_fetch": False, "historical_alpha": 0.3, "ada_param_enabled": adaptive})
    res = _launch(tmp_path, "tgn", None, "--ctdg-json", over)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    for r in range(2):
        o = _outcome(tmp_path, r)
        assert o["error"] is None and len(o["alphas"]) >= 2  # one per non-empty local step
        if adaptive:
            assert all(0.1 <= x <= 0.95 for x in o["alphas"]) and len(set(o["alphas"])) > 1
        else:
            assert set(o["alphas"]) == {0.3}


@pytest.mark.parametrize("remote_fetch", [True, False])
def test_ctdg_host_path_remote_reads(tmp_path, remote_fetch):
    """Remote reads on the host path: every step refreshes the rows it reads (roots and
    sampled neighbours) from their owners, in the same collective order on a step with
    no events; afterwards a pull of every remote row returns the owners' rows exactly.
    Without remote reads nothing is pulled."""
    res = _launch(tmp_path, "tgn", None, "--ctdg-json", json.dumps({"remote_fetch": remote_fetch}))
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    for r in range(2):
        o = _outcome(tmp_path, r)
        assert o["error"] is None
        if remote_fetch:
            assert o["pulled"] > 0 and o["pull_exact"]
        else:
            assert o["pulled"] == 0


def test_chunk_mode_two_ranks_uneven_clusters(tmp_path):
    """Three node clusters on two ranks: rank 0 runs two chunks per time slice, rank 1
    one. Both take the same number of steps (rank 1 pads with empty steps), so their
    collectives stay matched through train, validation, checkpoint and predict, and
    the replicas stay identical."""
    res = _launch(tmp_path, "tgn", None, "--chunk", "3")
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    o0, o1 = _outcome(tmp_path, 0), _outcome(tmp_path, 1)
    assert o0["error"] is None and o1["error"] is None
    assert o0["local_steps"] == o1["local_steps"] and o0["val_steps"] == o1["val_steps"]
    assert o0["own_chunks"] > o1["own_chunks"] > 0
    assert o0["local_steps"] >= o0["own_chunks"]  # a chunk runs as steps of at most batch_size events
    assert 0 < o1["engine_losses"] <= o0["engine_losses"] == o0["local_steps"]  # padding units carry no loss
    assert o0["predictions"] > 0
    p0, p1 = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    for a, b in zip(p0["params"], p1["params"]):
        assert torch.allclose(a, b, atol=1e-6)


def test_ctdg_exact_resume_two_ranks(tmp_path):
    """Each rank saves its own memory-bank rows, optimizer moments and random
    streams; a fresh session that loads them continues exactly like the
    uninterrupted run (losses, parameters, memory and mailbox on every rank)."""
    res = _launch(tmp_path, "tgn", None, "--resume")
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    for r in range(2):
        d = torch.load(tmp_path / f"resume_r{r}.pt")
        assert d["rank_file"]
        torch.testing.assert_close(torch.tensor(d["resumed"]), torch.tensor(d["full"]), rtol=0, atol=1e-6)
        for a, b in zip(d["params_full"], d["params_resumed"]):
            torch.testing.assert_close(a, b, rtol=0, atol=1e-6)
        torch.testing.assert_close(d["memory_resumed"], d["memory_full"], rtol=0, atol=1e-6)
        torch.testing.assert_close(d["mailbox_resumed"], d["mailbox_full"], rtol=0, atol=1e-6)


@pytest.mark.parametrize("world", [4, 8])
def test_many_ranks_dtdg_and_ctdg(tmp_path, world):
    """W = 4 and 8: every rank finishes the same number of steps with a finite
    loss and identical replicas (one all-reduced gradient per step), for the DTDG
    halo pipeline and the CTDG memory partition. At 8 ranks the small test graph
    leaves some partitions without rows in some snapshots."""
    for family in ("mpnn_lstm", "tgn"):
        out = tmp_path / family
        out.mkdir()
        res = _launch(out, family, nproc=world, wall=400)
        assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
        outs = [_outcome(out, r) for r in range(world)]
        assert all(o["error"] is None for o in outs)
        assert len({o["steps"] for o in outs}) == 1 and outs[0]["steps"] > 0
        assert all(math.isfinite(o["loss"]) for o in outs)
        ps = [torch.load(out / f"r{r}.pt") for r in range(world)]
        for r in range(1, world):
            for a, b in zip(ps[0]["params"], ps[r]["params"]):
                assert torch.allclose(a, b, atol=1e-6)


@pytest.mark.parametrize("family", ["tgcn", "evolvegcn", "jodie"])
def test_two_ranks_other_models(tmp_path, family):
    """The other models over two ranks: T-GCN (exchanges halo rows of its
    3 x hidden wide GCN layer), EvolveGCN (evolves replicated weights), JODIE
    (memory partitioned by owner, time-projection embedding)."""
    res = _launch(tmp_path, family)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    o0, o1 = _outcome(tmp_path, 0), _outcome(tmp_path, 1)
    assert o0["error"] is None and o1["error"] is None and o0["steps"] == o1["steps"] > 0
    assert math.isfinite(o0["loss"])
    p0, p1 = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    for a, b in zip(p0["params"], p1["params"]):
        assert torch.allclose(a, b, atol=1e-6)


def test_rank_exit_between_steps_is_detected(tmp_path):
    """Rank 1 exits before step 2; rank 0 must stop with an error (heartbeat or
    collective timeout) instead of waiting forever."""
    res = _launch(tmp_path, "mpnn_lstm", {"SU_FAULT": "1:2:exit"}, "--timeout", "20", "--heartbeat", "3",
                  wall=120)
    assert res.returncode != 0
    o0 = _outcome(tmp_path, 0)
    assert o0["error"] is not None, o0
    assert o0["elapsed_s"] < 90
    assert not (tmp_path / "outcome_r1.json").exists()  # rank 1 left without a word


def test_injected_exception_surfaces(tmp_path):
    res = _launch(tmp_path, "mpnn_lstm", {"SU_FAULT": "0:1:raise"}, "--timeout", "20", "--heartbeat", "3",
                  wall=120)
    assert res.returncode != 0
    o0 = _outcome(tmp_path, 0)
    assert o0["error"] == "InjectedFault"
    o1 = _outcome(tmp_path, 1)
    assert o1["error"] is not None  # the peer stops too (heartbeat or collective timeout)


@pytest.mark.parametrize("mode", ["dtdg", "ctdg", "chunk"])
def test_cli_all_phases_two_ranks(tmp_path, mode):
    """`python -m starry_unigraph --phase all` under torchrun with two gloo ranks:
    rank 0 writes the artifacts while the other waits, one process group serves
    prepare, train and predict, and the checkpoint is complete before any rank
    loads it."""
    import yaml

    family = "mpnn_lstm" if mode == "dtdg" else "tgn"
    cfg = {"model": {"name": family, "family": family, "hidden_dim": 16,
                     "task": "snapshot_node_regression" if mode == "dtdg" else "temporal_link_prediction"},
           "data": {"root": str(tmp_path / "data"), "name": f"cli_{mode}", "format": "mock"},
           "train": {"epochs": 2, "batch_size": 16, "snaps": 12},
           "runtime": {"device": "cpu", "checkpoint": str(tmp_path / "ckpt" / "cli" / "latest.pt")},
           "graph": {"storage": "snapshots" if mode == "dtdg" else "events"},
           "ctdg": {"dim_time": 8, "mailbox_slots": 1},
           "dist": {"backend": "gloo", "timeout_s": 120}}
    if mode == "chunk":
        cfg["data"].update({"format": "synthetic", "graph_mode": "chunk",
                            "synthetic": {"preset": "tgn_cpu", "num_events": 2000}})
        cfg["chunk"] = {"node_clusters": 3, "time_slices": 4}
    path = tmp_path / "cfg.yaml"
    path.write_text(yaml.safe_dump(cfg))
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    env.pop("CUDA_VISIBLE_DEVICES", None)
    for _ in range(3):  # a port picked free can be taken before the rendezvous binds it
        res = subprocess.run(["timeout", "-k", "10", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                              "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
                              "-m", "starry_unigraph", "--config", str(path), "--phase", "all",
                              "--artifact-root", str(tmp_path / "art")], cwd=tmp_path, env=env, capture_output=True,
                             text=True, timeout=360)
        if res.returncode == 0 or "Address already in use" not in res.stderr:
            break
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    assert res.stdout.count("epoch ") == 2 and "predict done" in res.stdout
    assert (tmp_path / "ckpt" / "cli" / "latest.pt").exists()


def test_comm_engine_two_ranks(tmp_path):
    """CommEngine (runtime/comm) on two gloo ranks: rows reach their owners, fetched
    rows equal the owners' rows, deltas are polled once, and the gradient all-reduce
    is the exact mean (int8: within one quantisation step)."""
    env = dict(os.environ)
    env.pop("CUDA_VISIBLE_DEVICES", None)
    worker = ROOT / "tests" / "workers" / "comm_engine_worker.py"
    for _ in range(3):  # a port picked free can be taken before the rendezvous binds it
        res = subprocess.run(["timeout", "-k", "10", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
                              "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_port()),
                              str(worker), "--out", str(tmp_path)], cwd=ROOT, env=env, capture_output=True, text=True,
                             timeout=300)
        if res.returncode == 0 or "Address already in use" not in res.stderr:
            break
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    for r in range(2):
        checks = json.loads((tmp_path / f"outcome_r{r}.json").read_text())
        assert all(checks.values()), checks


def test_ctdg_balanced_events_on_the_host_path(tmp_path):
    """event_partition: balanced on CPU ranks: each rank takes an equal share of every
    window (nodes it does not own included), pulls their rows from the owners and pushes
    the updates back; the replicas stay equal and the pulled rows match the owners'."""
    res = _launch(tmp_path, "tgn", None, "--ctdg-json", json.dumps({"event_partition": "balanced"}))
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-4000:]
    o0, o1 = _outcome(tmp_path, 0), _outcome(tmp_path, 1)
    assert o0["error"] is None and o1["error"] is None and o0["pulled"] > 0 and o0["pull_exact"] and o1["pull_exact"]
    p0, p1 = torch.load(tmp_path / "r0.pt"), torch.load(tmp_path / "r1.pt")
    for a, b in zip(p0["params"], p1["params"]):
        assert torch.allclose(a, b, atol=1e-6)
