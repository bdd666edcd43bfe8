"""SchedulerSession lifecycle on CPU (reference tests/test_session.py, rewritten for this API)."""
import json
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from starry_unigraph import SchedulerSession
from starry_unigraph.checkpoint import load_checkpoint

ROOT = Path(__file__).resolve().parents[1]


def make_config(tmp_path, family="tgn", task=None, **over):
    ctdg = family in ("tgn", "jodie", "dyrep", "tgat", "apan")
    cfg = {"model": {"name": family, "family": family,
                     "task": task or ("temporal_link_prediction" if ctdg else "snapshot_node_regression"),
                     "hidden_dim": 16},
           "data": {"root": str(tmp_path / "data"), "name": f"mock_{family}", "format": "mock"},
           "train": {"epochs": 1, "batch_size": 8, "snaps": 12},
           "runtime": {"device": "cpu", "checkpoint": str(tmp_path / "ckpt" / "latest.pt")},
           "graph": {"storage": "events" if ctdg else "snapshots"},
           "ctdg": {"dim_time": 8, "mailbox_slots": 2}}
    for k, v in over.items():
        cfg.setdefault(k, {}).update(v)
    return cfg


def _session(tmp_path, **kw):
    s = SchedulerSession.from_config(make_config(tmp_path, **kw))
    s.ctx.artifact_root = tmp_path / "artifacts"
    return s


@pytest.mark.parametrize("family", ["tgn", "jodie", "dyrep", "tgat", "apan"])
def test_ctdg_prepare_train_eval_predict(tmp_path, family):
    s = _session(tmp_path, family=family)
    prepared = s.prepare_data()
    meta = json.loads(prepared.meta_path.read_text())
    assert meta["graph_mode"] == "ctdg" and meta["artifact_version"] == 1
    for rel in ("partitions/manifest.json", "routes/manifest.json", "sampling/index.json"):
        assert (s.ctx.artifact_root / rel).exists()
    s.build_runtime()
    r = s.run_epoch("train")
    assert set(r) >= {"split", "steps", "local_steps", "loss", "local_loss", "metrics", "elapsed_s",
                      "local_elapsed_s", "outputs"}
    assert r["steps"] > 0 and r["loss"] > 0
    v = s.evaluate("val")
    assert v["steps"] > 0
    p = s.predict("test")
    assert len(p.predictions) > 0 and p.meta["graph_mode"] == "ctdg"


@pytest.mark.parametrize("family", ["mpnn_lstm", "tgcn", "evolvegcn", "gcn"])
def test_dtdg_prepare_train_eval_predict(tmp_path, family):
    s = _session(tmp_path, family=family)
    s.prepare_data()
    for rel in ("flare/manifest.json", "flare/part_000.pth", "partitions/manifest.json", "routes/manifest.json"):
        assert (s.ctx.artifact_root / rel).exists()
    s.build_runtime()
    assert s.runtime.state["graph_mode"] == "dtdg"
    r = s.run_epoch("train")
    assert r["steps"] > 0 and r["loss"] >= 0
    v = s.run_epoch("val")
    assert v["steps"] >= 1
    p = s.predict("test")
    assert len(p.predictions) > 0 and p.targets is not None


def test_run_task(tmp_path):
    s = _session(tmp_path, family="mpnn_lstm")
    s.prepare_data()
    out = s.run_task()
    assert out["epochs"] == 1 and len(out["train"]) == 1 and len(out["eval"]) == 1


def test_ctdg_checkpoint_roundtrip(tmp_path):
    s = _session(tmp_path)
    s.prepare_data()
    s.build_runtime()
    s.run_epoch("train")
    path = s.save_checkpoint(tmp_path / "c.pt", exact_resume=True)
    ck = torch.load(path, weights_only=False)
    assert set(ck) >= {"model", "memory_updater", "exact_resume"}
    rank_state = load_checkpoint(s.rank_state_path(path, 0))
    assert set(rank_state) >= {"memory_bank", "optimizer", "rng"}
    s2 = _session(tmp_path)
    s2.prepared = None
    s2.ctx.artifact_root = s.ctx.artifact_root
    s2.build_runtime()
    torch.manual_seed(12345)  # a different RNG position than at save time
    s2.load_checkpoint(path)
    for a, b in zip(s.runtime.model.state_dict().values(), s2.runtime.model.state_dict().values()):
        assert torch.equal(a, b)
    # exact resume: memory bank, optimizer moments, RNG stream and counters come back
    for n in ("memory", "memory_ts", "mailbox", "mailbox_ts"):
        assert torch.equal(getattr(s.ctdg_session.online_runtime.memory, n).cpu(),
                           getattr(s2.ctdg_session.online_runtime.memory, n).cpu())
    st1, st2 = s.runtime.optimizer.state_dict()["state"], s2.runtime.optimizer.state_dict()["state"]
    assert st1.keys() == st2.keys() and len(st1) > 0
    for k in st1:
        assert torch.equal(st1[k]["exp_avg"], st2[k]["exp_avg"])
    assert torch.equal(torch.get_rng_state(), rank_state["rng"]["torch"])
    assert s2.global_step == s.global_step and s2.current_epoch == s.current_epoch


def test_dtdg_checkpoint_roundtrip(tmp_path):
    s = _session(tmp_path, family="tgcn")
    s.prepare_data()
    s.build_runtime()
    s.run_epoch("train")
    path = s.save_checkpoint(tmp_path / "d.pt")
    import pickle

    with open(path, "rb") as handle:  # the reference's loader is a plain pickle.load
        payload = pickle.load(handle)
    assert set(payload) >= {"model_state", "optimizer_state", "scheduler_state", "config", "epoch", "global_step"}
    s2 = _session(tmp_path, family="tgcn")
    s2.ctx.artifact_root = s.ctx.artifact_root
    s2.load_checkpoint(path)
    assert s2.current_epoch == 1
    for a, b in zip(s.runtime.model.state_dict().values(), s2.runtime.model.state_dict().values()):
        assert torch.equal(a, b)


def test_artifact_validation(tmp_path):
    from starry_unigraph.session import validate_artifacts

    s = _session(tmp_path, family="mpnn_lstm")
    prepared = s.prepare_data()
    validate_artifacts(prepared, "dtdg", 1)
    with pytest.raises(RuntimeError):
        validate_artifacts(prepared, "ctdg", 1)
    with pytest.raises(RuntimeError):
        validate_artifacts(prepared, "dtdg", 2)
    meta = json.loads(prepared.meta_path.read_text())
    meta["artifact_version"] = 99
    prepared.meta_path.write_text(json.dumps(meta))
    with pytest.raises(RuntimeError):
        validate_artifacts(prepared, "dtdg", 1)


def test_build_runtime_without_prepare_raises(tmp_path):
    s = _session(tmp_path)
    with pytest.raises(RuntimeError):
        s.build_runtime()


def test_node_classification_dtdg(tmp_path):
    cfg = make_config(tmp_path, family="tgcn", task="node_classification")
    cfg["data"] = {"root": str(tmp_path), "name": "cls", "format": "synthetic",
                   "synthetic": {"num_nodes": 300, "num_snapshots": 6, "edges_per_snapshot": 1500, "churn": 0.1,
                                 "feat_dim": 8, "label": "binary"}}
    s = SchedulerSession.from_config(cfg)
    s.ctx.artifact_root = tmp_path / "a"
    s.prepare_data()
    s.build_runtime()
    r = s.run_epoch("train")
    assert r["loss"] > 0


def test_cli_prepare_train_predict(tmp_path):
    import yaml

    cfg = make_config(tmp_path, family="mpnn_lstm")
    path = tmp_path / "cfg.yaml"
    path.write_text(yaml.safe_dump(cfg))
    env = {"PYTHONPATH": str(ROOT), "PATH": "/usr/bin:/bin"}
    for phase in ("prepare", "train", "predict"):
        out = subprocess.run([sys.executable, "-m", "starry_unigraph", "--config", str(path), "--phase", phase,
                              "--artifact-root", str(tmp_path / "art")], capture_output=True, text=True,
                             cwd=tmp_path, env=env, timeout=300)
        assert out.returncode == 0, out.stderr[-2000:]
    assert "MAE=" in out.stdout


def test_subcommand_cli(tmp_path, monkeypatch, capsys):
    """`starry-unigraph --config CFG prepare|train|predict|resume` (reference cli/main.py)."""
    import yaml

    from starry_unigraph.cli.main import main as cli_main

    monkeypatch.chdir(tmp_path)  # artifacts land under ./artifacts/<data.name>
    cfg = make_config(tmp_path, family="tgn")
    path = tmp_path / "cfg.yaml"
    path.write_text(yaml.safe_dump(cfg))
    for argv in (["prepare"], ["train"], ["predict", "--split", "val"]):
        assert cli_main(["--config", str(path), *argv]) == 0
    lines = [json.loads(x) for x in capsys.readouterr().out.splitlines() if x.startswith("{")]
    assert [x["command"] for x in lines] == ["prepare", "train", "predict"]
    assert lines[1]["epochs"] == 1 and lines[2]["predictions"] > 0
    s = SchedulerSession.from_config(cfg)
    s.build_runtime()
    s.run_epoch("train")
    ckpt = s.save_checkpoint(tmp_path / "ckpt" / "resume.pt")
    assert cli_main(["--config", str(path), "resume", "--checkpoint", str(ckpt)]) == 0
    assert json.loads(capsys.readouterr().out.splitlines()[-1])["command"] == "resume"


def test_cuda_step_batch_capacity_from_artifacts(tmp_path):
    """With the owner rule the CUDA step's buffers hold the largest per-rank share of a
    global window: taken from the artifacts' metadata when another process prepared
    them (a CLI train phase after its prepare phase), not guessed."""
    from types import SimpleNamespace

    from starry_unigraph.backends.ctdg.runtime.factory import _engine_bmax

    meta = SimpleNamespace(provider_meta={"max_local_batch": 37})
    ctx = SimpleNamespace(provider_state={}, prepared_artifacts=meta)
    assert _engine_bmax(ctx, 20, 2, True) == 37
    assert _engine_bmax(ctx, 20, 1, True) == 20 and _engine_bmax(ctx, 20, 2, False) == 20
    ctx.provider_state["max_local_batch"] = 41
    assert _engine_bmax(ctx, 20, 2, True) == 41
    assert _engine_bmax(SimpleNamespace(provider_state={}, prepared_artifacts=None), 20, 2, True) == 40
    # the preprocessor records it for several ranks
    s = _session(tmp_path, family="tgn", dist={"world_size": 2})
    prepared = s.prepare_data()
    assert prepared.provider_meta["max_local_batch"] >= 1


def test_dtdg_eval_metrics_follow_the_task(tmp_path):
    """Classification runs report accuracy, regression runs MAE / RMSE."""
    from starry_unigraph.backends.dtdg.runtime.training import _eval_metrics

    assert _eval_metrics("node_classification", torch.tensor([2.0, -1.0, 0.5]), torch.tensor([1, 0, 0])) == \
        {"accuracy": pytest.approx(2 / 3)}
    logits = torch.tensor([[0.1, 0.9], [0.8, 0.2]]).view(-1)
    assert _eval_metrics("node_classification", logits, torch.tensor([1, 1]))["accuracy"] == pytest.approx(0.5)
    m = _eval_metrics("snapshot_node_regression", torch.tensor([1.0, 3.0]), torch.tensor([2.0, 3.0]))
    assert m["mae"] == pytest.approx(0.5) and m["rmse"] == pytest.approx(0.5 ** 0.5)
    cfg = make_config(tmp_path, family="tgcn", task="node_classification")
    s = SchedulerSession.from_config(cfg)
    s.ctx.artifact_root = tmp_path / "art"
    s.prepare_data()
    s.build_runtime()
    s.run_epoch("train")
    assert "accuracy" in s.run_epoch("val")["metrics"]


def test_metrics_jsonl(tmp_path):
    """runtime.metrics_path: one JSON line per epoch summary with the losses and metrics."""
    path = tmp_path / "m" / "metrics.jsonl"
    s = _session(tmp_path, family="tgn", runtime={"metrics_path": str(path)})
    s.prepare_data()
    s.build_runtime()
    s.run_epoch("train")
    s.run_epoch("val")
    rows = [json.loads(x) for x in path.read_text().splitlines()]
    assert [r["split"] for r in rows] == ["train", "val"]
    assert all({"epoch", "steps", "loss", "global_loss", "metrics", "elapsed_s"} <= set(r) for r in rows)
    assert rows[0]["loss"] > 0 and "auc" in rows[1]["metrics"]
