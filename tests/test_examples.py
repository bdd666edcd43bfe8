"""User configs (configs/*.yaml) and example scripts (examples/*.py) on CPU: every config
loads and validates for its model family, each example trains, checkpoints and tests a
shrunken version of its workload, chunk mode runs through the CLI, and a two-rank gloo run
of the DTDG example reports the same global loss as one rank (reference configs/ and
examples/ directories)."""
import importlib.util
import os
import re
import socket
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
CONFIGS = sorted((ROOT / "configs").glob("*.yaml"))


def _example(name):
    spec = importlib.util.spec_from_file_location(f"example_{name}", ROOT / "examples" / f"{name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("path", CONFIGS, ids=[p.stem for p in CONFIGS])
def test_config_loads_and_validates(path):
    from starry_unigraph.config.schema import detect_graph_mode, load_config, validate_config
    from starry_unigraph.registry import ModelRegistry, TaskRegistry

    cfg = load_config(path)
    assert validate_config(cfg) == []  # no missing path, no field inactive for the mode
    spec = ModelRegistry.resolve(model_name=cfg["model"]["name"], family=cfg["model"]["family"])
    TaskRegistry.resolve(cfg["model"]["task"])
    mode = detect_graph_mode(cfg)
    assert mode == "chunk" or spec.graph_mode == mode
    assert cfg["dist"]["master_addr"] == "127.0.0.1"


def test_configs_cover_every_benchmark_family():
    from starry_unigraph.config.schema import load_config

    families = {load_config(p)["model"]["family"] for p in CONFIGS}
    assert families >= {"tgn", "jodie", "mpnn_lstm", "tgcn", "evolvegcn"}


def test_tgn_example_trains_checkpoints_and_tests(tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)  # the config's checkpoint path is relative
    res = _example("train_tgn").main(["--config", str(ROOT / "configs" / "tgn_large_nvlink.yaml"), "--device", "cpu",
                                      "--events", "4000", "--batch-size", "400", "--epochs", "2",
                                      "--artifact-root", str(tmp_path / "art"), "--exact-resume"])
    assert set(res["test"]) == {"ap", "auc", "mrr"} and 0.0 <= res["test"]["ap"] <= 1.0
    assert (tmp_path / "checkpoints" / "tgn_large" / "latest.pt").exists()
    assert (tmp_path / "checkpoints" / "tgn_large" / "latest.pt.rank0").exists()  # exact-resume state
    # continue from the exact-resume checkpoint
    again = _example("train_tgn").main(["--config", str(ROOT / "configs" / "tgn_large_nvlink.yaml"), "--device", "cpu",
                                        "--events", "4000", "--batch-size", "400", "--epochs", "1", "--mode", "train",
                                        "--artifact-root", str(tmp_path / "art"),
                                        "--resume", str(tmp_path / "checkpoints" / "tgn_large" / "latest.pt")])
    assert again["train_loss"] > 0


@pytest.mark.parametrize("config,task_key", [("mpnn_lstm_nvlink", "rmse"), ("tgcn_large", "accuracy"),
                                             ("evolvegcn_large", "accuracy")])
def test_dtdg_example_trains_and_tests(tmp_path, monkeypatch, config, task_key):
    monkeypatch.chdir(tmp_path)
    res = _example("train_mpnn_lstm").main(["--config", str(ROOT / "configs" / f"{config}.yaml"), "--device", "cpu",
                                            "--epochs", "1", "--nodes", "1500", "--edges", "12000",
                                            "--snapshots", "12", "--artifact-root", str(tmp_path / "art")])
    assert res["train_loss"] > 0 and task_key in res["test"]


def test_chunk_config_through_cli(tmp_path):
    cmd = [sys.executable, "-m", "starry_unigraph", "--config", str(ROOT / "configs" / "chunk_default.yaml"),
           "--device", "cpu", "--epochs", "1", "--artifact-root", str(tmp_path / "art")]
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    res = subprocess.run(cmd, cwd=tmp_path, env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-3000:]
    assert "train_loss=" in res.stdout and "predict done" in res.stdout


def _train_losses(text):
    return [float(m) for m in re.findall(r"train loss ([0-9.]+)", text)]


def test_dtdg_example_two_gloo_ranks_match_one_rank(tmp_path):
    """Nodes split over two ranks, one gradient all-reduce per step: the global loss of each
    epoch is the one-rank loss (both runs start from the same seed and data)."""
    args = ["--config", str(ROOT / "configs" / "mpnn_lstm_nvlink.yaml"), "--device", "cpu", "--backend", "gloo",
            "--epochs", "2", "--nodes", "2000", "--edges", "16000", "--snapshots", "12", "--mode", "all"]
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    env.pop("CUDA_VISIBLE_DEVICES", None)
    one = subprocess.run([sys.executable, str(ROOT / "examples" / "train_mpnn_lstm.py"), *args,
                          "--artifact-root", str(tmp_path / "a1")], cwd=tmp_path, env=env, capture_output=True,
                         text=True, timeout=600)
    assert one.returncode == 0, one.stderr[-3000:]
    for _ in range(3):  # a port picked free can be taken before the rendezvous binds it
        two = subprocess.run(["timeout", "-k", "10", "420", sys.executable, "-m", "torch.distributed.run",
                              "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port",
                              str(_port()), str(ROOT / "examples" / "train_mpnn_lstm.py"), *args,
                              "--artifact-root", str(tmp_path / "a2")], cwd=tmp_path, env=env, capture_output=True,
                             text=True, timeout=480)
        if two.returncode == 0 or "Address already in use" not in two.stderr:
            break
    assert two.returncode == 0, two.stdout[-2000:] + two.stderr[-3000:]
    l1, l2 = _train_losses(one.stdout), _train_losses(two.stdout)
    assert len(l1) == len(l2) == 2
    assert l1 == pytest.approx(l2, rel=1e-4)


def test_custom_model_through_the_engine_learns(tmp_path, monkeypatch):
    """A user model on materialised batches with neighbour feature rows (the engine given
    a feature store) trains through PipelineEngine to a validation AUC above 0.6."""
    monkeypatch.chdir(tmp_path)
    torch = pytest.importorskip("torch")
    torch.manual_seed(0)
    res = _example("custom_model_engine").main(["--config", str(ROOT / "configs" / "tgn_large_nvlink.yaml"),
                                                "--events", "8000", "--batch-size", "400", "--epochs", "3",
                                                "--artifact-root", str(tmp_path / "art")])
    assert res["train"] and res["val"]["metrics"]["auc"] > 0.6


def test_multi_gpu_launcher_on_gloo_ranks(tmp_path):
    """examples/run_multi_gpu.sh (one torchrun call over all phases) on two CPU ranks."""
    import yaml

    cfg = {"model": {"name": "mpnn_lstm", "family": "mpnn_lstm", "task": "snapshot_node_regression",
                     "hidden_dim": 16},
           "data": {"root": str(tmp_path / "data"), "name": "launcher", "format": "mock"},
           "train": {"epochs": 1, "snaps": 12},
           "runtime": {"device": "cpu", "checkpoint": str(tmp_path / "ckpt" / "x" / "latest.pt")},
           "graph": {"storage": "snapshots"}, "dist": {"backend": "gloo", "timeout_s": 120}}
    (tmp_path / "c.yaml").write_text(yaml.safe_dump(cfg))
    env = dict(os.environ, LOG_DIR=str(tmp_path / "logs"), WALL_S="300")
    env.pop("CUDA_VISIBLE_DEVICES", None)
    for _ in range(3):  # a port picked free can be taken before the rendezvous binds it
        env["PORT"] = str(_port())
        res = subprocess.run(["bash", str(ROOT / "examples" / "run_multi_gpu.sh"), str(tmp_path / "c.yaml"), "2", "all",
                              "--artifact-root", str(tmp_path / "art")], cwd=tmp_path, env=env, capture_output=True,
                             text=True, timeout=360)
        if res.returncode == 0 or "Address already in use" not in res.stdout + res.stderr:
            break
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    assert "predict done" in res.stdout and list((tmp_path / "logs").glob("*.log"))


def test_tgn_example_two_gloo_ranks(tmp_path):
    """The CTDG example under torchrun: rank 0 prepares, both ranks train, checkpoint and test."""
    args = ["--config", str(ROOT / "configs" / "tgn_large_nvlink.yaml"), "--device", "cpu", "--backend", "gloo",
            "--events", "4000", "--batch-size", "200", "--epochs", "1", "--artifact-root", str(tmp_path / "art")]
    env = dict(os.environ, PYTHONPATH=str(ROOT))
    env.pop("CUDA_VISIBLE_DEVICES", None)
    for _ in range(3):  # a port picked free can be taken before the rendezvous binds it
        res = subprocess.run(["timeout", "-k", "10", "420", sys.executable, "-m", "torch.distributed.run",
                              "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port",
                              str(_port()), str(ROOT / "examples" / "train_tgn.py"), *args], cwd=tmp_path, env=env,
                             capture_output=True, text=True, timeout=480)
        if res.returncode == 0 or "Address already in use" not in res.stderr:
            break
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-3000:]
    assert "events/s" in res.stdout and "[test]" in res.stdout
    assert (tmp_path / "checkpoints" / "tgn_large" / "latest.pt").exists()
