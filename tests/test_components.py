"""Chunk mode, the unified pipeline engine, caches, comm engine and the stable
library surface, on CPU (reference tests/test_chunk_pipeline.py,
tests/test_lib_api.py, tests/test_engine.py)."""
import torch

from starry_unigraph import SchedulerSession

from test_session import make_config


def _chunk_session(tmp_path):
    cfg = make_config(tmp_path, family="tgn")
    cfg["data"]["graph_mode"] = "chunk"
    cfg["chunk"] = {"node_clusters": 4, "time_slices": 4}
    s = SchedulerSession.from_config(cfg)
    s.ctx.artifact_root = tmp_path / "artifacts"
    return s


def test_chunk_mode_lifecycle(tmp_path):
    s = _chunk_session(tmp_path)
    s.prepare_data()
    for rel in ("snapshots/manifest.json", "clusters/part_000/cluster_manifest.json", "clusters/part_000/chunks.pt"):
        assert (s.ctx.artifact_root / rel).exists()
    s.build_runtime()
    assert s.runtime.state["graph_mode"] == "chunk"
    r = s.run_epoch("train")
    assert r["steps"] > 0 and r["loss"] > 0
    assert s.run_epoch("val")["steps"] > 0
    assert len(s.predict("test").predictions) > 0


def test_pipeline_engine_epoch(tmp_path):
    s = _chunk_session(tmp_path)
    s.prepare_data()
    eng = s.build_pipeline_engine()
    out = eng.run_epoch("train", batch_size=8)
    assert set(out) >= {"split", "loss", "num_batches", "metrics", "outputs"}


def test_hot_and_decay_caches():
    from starry_unigraph.runtime.cache.decay_cache import DecayCache
    from starry_unigraph.runtime.cache.hot_cache import HotCache

    hc = HotCache(4, 3)
    hc.insert(torch.tensor([1, 2]), torch.arange(6.0).view(2, 3))
    hit, rows = hc.lookup(torch.tensor([2, 5]))
    assert hit.tolist() == [True, False] and torch.equal(rows[0], torch.tensor([3.0, 4.0, 5.0]))
    dc = DecayCache(max_versions=2)
    for v in range(4):
        dc.put(v, torch.tensor([v]), torch.ones(1, 2) * v)
        dc.expire(v)
    assert dc.get(0) is None and dc.get(3) is not None


def test_comm_engine_single_process():
    from starry_unigraph.runtime.comm.comm_engine import CommEngine

    ce = CommEngine()
    table = torch.arange(6.0).view(3, 2)
    assert torch.equal(ce.async_fetch(torch.tensor([2, 0]), table).wait(), table[[2, 0]])


def test_stable_api_surface():
    import starry_unigraph.lib_stable as L

    for name in L.__all__:
        assert hasattr(L, name), name
    assert "stable" in L.get_stability_info()


def test_native_sampler_wrapper():
    from starry_unigraph.native import BTSNativeSampler, build_temporal_neighbor_block, is_bts_sampler_available

    assert is_bts_sampler_available()
    row = torch.tensor([0, 1, 2, 0, 3])
    col = torch.tensor([1, 2, 3, 3, 1])
    ts = torch.tensor([1, 2, 3, 4, 5])
    tnb = build_temporal_neighbor_block("wrapper_test", row, col, 4, torch.arange(5), timestamp=ts)
    smp = BTSNativeSampler(tnb, num_nodes=4, num_edges=5, num_layers=1, fanout=[2], policy="recent")
    ret = smp.sample_from_nodes(torch.tensor([3, 1]), torch.tensor([10, 10]))
    assert len(ret) == 1
