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


def _stream(n_nodes=60, n_events=800, seed=0):
    g = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n_nodes, (n_events,), generator=g)
    dst = torch.randint(0, n_nodes, (n_events,), generator=g)
    ts = torch.sort(torch.rand(n_events, generator=g) * 1000).values
    return src, dst, ts, n_nodes


def test_chunk_dependence_routes_and_schedule():
    """Temporal routes: same cluster, earlier slices, newest first, decay^k
    weights; spatial routes: clusters joined by an event of the same slice;
    the schedule runs every chunk after its temporal dependencies."""
    from starry_unigraph.backends.chunk.prepare import ChunkGenerator, schedule

    src, dst, ts, n = _stream()
    gen = ChunkGenerator(num_clusters=3, time_slices=4, adaptive=False, decay_base=0.5)
    out = gen.generate(src, dst, ts, n)
    cluster, routes = out["clusters"], out["routes"]
    ids = {r.chunk_id for r in routes}
    slice_of = torch.arange(src.numel()) // ((src.numel() + 3) // 4)
    for r in routes:
        t, c = r.chunk_id
        expect_t = sorted((s for s, cc in ids if cc == c and s < t), reverse=True)
        assert r.temporal_deps == [(s, c) for s in expect_t]
        assert torch.allclose(r.decay_weights, 0.5 ** torch.arange(1, len(expect_t) + 1, dtype=torch.float32))
        m = slice_of == t
        a, b = cluster[src[m]], cluster[dst[m]]
        linked = set(b[a == c].tolist()) | set(a[b == c].tolist())
        assert set(d[1] for d in r.gnn_deps) == {x for x in linked if x != c and (t, x) in ids}
    order = schedule(routes)
    pos = {cid: i for i, cid in enumerate(order)}
    assert len(order) == len(routes)
    assert all(pos[d] < pos[r.chunk_id] for r in routes for d in r.temporal_deps)


def test_adaptive_cluster_count_grows_with_cross_traffic():
    from starry_unigraph.backends.chunk.prepare import ChunkGenerator

    src, dst, ts, n = _stream(n_nodes=200, n_events=3000, seed=1)  # random graph: most events cross clusters
    fixed = ChunkGenerator(num_clusters=2, adaptive=False)
    grown = ChunkGenerator(num_clusters=2, adaptive=True, info_loss_threshold=0.2)
    _, n_fixed, r_fixed = fixed.generate_graph_clusters(src, dst, n)
    _, n_grown, _ = grown.generate_graph_clusters(src, dst, n)
    assert n_fixed == 2 and r_fixed > 0.2
    import math

    assert n_grown == math.ceil(2 * r_fixed / 0.2)


def test_chunk_artifacts_carry_routes_and_order(tmp_path):
    import json

    s = _chunk_session(tmp_path)
    s.prepare_data()
    routes = json.loads((s.ctx.artifact_root / "routes" / "manifest.json").read_text())
    assert routes["dependence_routes"] and routes["order"]
    s.build_runtime()
    order = [tuple(c) for c in routes["order"]]
    mine = [c.chunk_id for c in s.snapshot_core._splits["train"]]
    ranks = [order.index(tuple(c)) for c in mine]
    assert ranks == sorted(ranks)


def test_historical_cache_threshold_and_adaptive_alpha():
    """A shared node is pushed when its cosine distance to the last pushed row exceeds
    1 - alpha; sync-heavy steps lower alpha (fewer pushes), compute-heavy steps raise it."""
    from starry_unigraph.backends.ctdg.runtime.cache import AdaParameter, CTDGHistoricalCache

    shared = torch.tensor([1, 3, 5])
    cache = CTDGHistoricalCache(3, 2, "cpu", num_nodes=6, shared_node_ids=shared, ada_param=AdaParameter(alpha=0.5))
    ids = torch.tensor([1, 3, 5, 0])
    rows = torch.tensor([[1.0, 0.0], [1.0, 0.0], [1.0, 0.0], [1.0, 0.0]])
    assert cache.historical_check(ids, rows).tolist() == [True, True, True, True]  # never cached / not shared
    cache.update_cache(cache.slot_indices(ids[:3]), rows[:3], torch.zeros(3))
    # cosine distances 0, 1 - cos(60 deg) = 0.5, 1 - cos(90 deg) = 1 against the threshold 0.5
    new = torch.tensor([[1.0, 0.0], [0.5, 0.75 ** 0.5 + 1e-3], [0.0, 1.0], [1.0, 0.0]])
    assert cache.historical_check(ids, new).tolist() == [False, True, True, True]
    ada = cache.ada_param
    ada.update_from_latency(sync_ms=30.0, compute_ms=10.0)  # sync dominates
    assert ada.alpha < 0.5
    assert cache.historical_check(ids, new).tolist() == [False, False, True, True]
    for _ in range(1000):
        ada.update_from_latency(sync_ms=0.0, compute_ms=10.0)
    assert ada.alpha == ada.max_alpha
    for _ in range(1000):
        ada.update_from_latency(sync_ms=1e3, compute_ms=1.0)
    assert ada.alpha == ada.min_alpha
