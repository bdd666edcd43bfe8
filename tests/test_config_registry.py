"""Config schema, registries, split bounds, task adapters (reference tests/test_session.py:189-229,
tests/test_orthogonal_separation.py)."""
import pytest
import torch

from starry_unigraph.config.schema import ConfigError, detect_graph_mode, load_config, validate_config
from starry_unigraph.distributed import DistRouteIndex, apply_distributed_env, build_distributed_context
from starry_unigraph.registry import ModelRegistry, TaskRegistry
from starry_unigraph.runtime._split import normalize_split_ratio, split_bounds


def test_load_config_merges_defaults_and_overrides():
    cfg = load_config({"model": {"name": "tgn", "family": "tgn"}}, overrides={"train": {"epochs": 7}})
    assert cfg["train"]["epochs"] == 7
    assert cfg["train"]["batch_size"] == 32
    assert cfg["dist"]["backend"] == "nccl"


def test_graph_mode_inference():
    for fam, mode in [("tgn", "ctdg"), ("jodie", "ctdg"), ("mpnn_lstm", "dtdg"), ("evolvegcn", "dtdg"),
                      ("gcn", "dtdg")]:
        cfg = load_config({"model": {"name": fam, "family": fam}})
        assert detect_graph_mode(cfg) == mode


def test_missing_required_path_raises():
    cfg = load_config({})
    del cfg["train"]["epochs"]
    with pytest.raises(ConfigError):
        validate_config(cfg)


def test_inactive_field_warning():
    cfg = load_config({"model": {"name": "mpnn_lstm", "family": "mpnn_lstm"}, "graph": {"storage": "snapshots"},
                       "sampling": {"neighbor_limit": [5]}})
    warnings = validate_config(cfg)
    assert any("sampling.neighbor_limit" in w for w in warnings)


def test_torchrun_env_overrides(monkeypatch):
    monkeypatch.setenv("WORLD_SIZE", "4")
    monkeypatch.setenv("RANK", "2")
    monkeypatch.setenv("LOCAL_RANK", "1")
    cfg = apply_distributed_env(load_config({"runtime": {"device": "cuda"}}))
    ctx = build_distributed_context(cfg)
    assert (ctx.world_size, ctx.rank, ctx.local_rank, ctx.launcher) == (4, 2, 1, "torchrun")
    assert cfg["runtime"]["device"] == "cuda:1"


def test_registries():
    assert ModelRegistry.resolve(family="TGN").graph_mode == "ctdg"
    assert ModelRegistry.resolve(model_name="mpnn_lstm").graph_mode == "dtdg"
    with pytest.raises(KeyError):
        ModelRegistry.resolve(family="nope")
    assert set(TaskRegistry.list_tasks()) >= {"temporal_link_prediction", "edge_predict", "snapshot_node_regression",
                                              "node_regression", "node_classification"}


@pytest.mark.parametrize("total", [0, 1, 2, 3, 10, 101, 157474])
def test_split_bounds_cover_and_nonempty(total):
    r = normalize_split_ratio({"train": 0.7, "val": 0.15, "test": 0.15})
    b = [split_bounds(total, s, r) for s in ("train", "val", "test")]
    assert b[0][0] == 0 and b[2][1] == total
    assert b[0][1] == b[1][0] and b[1][1] == b[2][0]
    if total >= 3:
        assert all(e > s for s, e in b)


def test_dist_route_index_roundtrip():
    idx = DistRouteIndex(torch.tensor([5, 7, 1 << 40]), torch.tensor([3, 0, 16383]))
    assert idx.loc.tolist() == [5, 7, 1 << 40]
    assert idx.part.tolist() == [3, 0, 16383]
    idx.set_shared(torch.tensor([1]))
    assert idx.is_shared.tolist() == [False, True, False]


def test_task_adapters():
    from starry_unigraph.tasks import EdgePredictAdapter, NodeClassifyAdapter, NodeRegressionTaskAdapter
    from starry_unigraph.data.batch_data import BatchData

    ep = EdgePredictAdapter()
    out = {"pos_score": torch.tensor([2.0, 3.0]), "neg_score": torch.tensor([-1.0, 0.5])}
    assert float(ep.compute_loss(out)) > 0
    m = ep.compute_metrics(out)
    assert m["auc"] == 1.0 and m["ap"] == 1.0
    nr = NodeRegressionTaskAdapter()
    b = BatchData(mfg=None, node_ids=torch.arange(3), labels=torch.tensor([1.0, 2.0, 3.0]))
    assert abs(float(nr.compute_loss({"predictions": torch.tensor([1.0, 2.0, 4.0])}, b)) - 1 / 3) < 1e-6
    nc = NodeClassifyAdapter()
    assert nc.compute_metrics({"logits": torch.tensor([[2.0, 0.0], [0.0, 1.0]])},
                              BatchData(mfg=None, node_ids=torch.arange(2), labels=torch.tensor([0, 1])))["accuracy"] == 1
    assert ep.compute_loss({"loss": 0.25}) == 0.25


def test_heads_and_wrapped_model():
    from starry_unigraph.data.batch_data import BatchData
    from starry_unigraph.models import EdgePredictHead, NodeRegressHead, WrappedModel

    class Backbone(torch.nn.Module):
        def forward(self, mfg, state):
            return torch.ones(4, 3)

    w = WrappedModel(Backbone(), EdgePredictHead(3))
    out = w({}, BatchData(mfg=None, node_ids=torch.arange(4), pos_src=torch.tensor([0]), pos_dst=torch.tensor([1]),
                          neg_src=torch.tensor([2]), neg_dst=torch.tensor([3])))
    assert out["pos_score"].tolist() == [3.0]
    r = NodeRegressHead(3)(torch.ones(4, 3), BatchData(mfg=None, node_ids=torch.arange(4), target_nodes=torch.tensor([0, 2])))
    assert r["node_pred"].shape == (2, 1)


def test_config_reference_covers_every_default_key():
    """docs/config.md names every key of default.yaml (by dotted path, a `section.*`
    wildcard, or its leaf name in its section's table)."""
    from pathlib import Path

    from starry_unigraph.config.schema import load_default_config

    doc = (Path(__file__).resolve().parents[1] / "docs" / "config.md").read_text()
    sections = {}
    for block in doc.split("\n## ")[1:]:
        title, _, body = block.partition("\n")
        sections[title.strip()] = body

    def leaves(d, prefix=""):
        for k, v in d.items():
            path = f"{prefix}{k}"
            if isinstance(v, dict) and v:
                yield from leaves(v, path + ".")
            else:
                yield path

    missing = []
    for path in leaves(load_default_config()):
        top, leaf = path.split(".")[0], path.split(".")[-1]
        wild = ".".join(path.split(".")[:2]) + ".*"
        body = next((b for t, b in sections.items() if top in t.split()), "")
        parts = path.split(".")
        # the path below its section, or an ancestor of it, named in the section's table
        named = any(f"`{'.'.join(parts[1:j])}`" in body for j in range(2, len(parts) + 1))
        if path not in doc and wild not in doc and f"`{leaf}`" not in body and not named:
            missing.append(path)
    assert not missing, missing
