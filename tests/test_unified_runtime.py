"""Unified-runtime pieces on CPU: the hot cache (vectorised insert), the CTDG /
DTDG state managers, the runners driven through the session, the spatial /
state communication plans and the route volume summary the DTDG session
records."""
import pytest
import torch

from starry_unigraph import SchedulerSession
from starry_unigraph.runtime.cache import DecayCache, HotCache
from starry_unigraph.runtime.comm.spatial_plan import SpatialPlan
from starry_unigraph.runtime.comm.state_plan import StatePlan
from starry_unigraph.runtime.runner import run_units


def test_hot_cache_insert_and_lookup():
    torch.manual_seed(0)
    cache = HotCache(capacity=8, dim=4)
    ids = torch.tensor([5, 3, 5, 9])      # repeated id: the last row wins
    rows = torch.arange(16, dtype=torch.float32).view(4, 4)
    cache.insert(ids, rows)
    hit, got = cache.lookup(torch.tensor([5, 3, 9, 7]))
    assert hit.tolist() == [True, True, True, False]
    assert torch.equal(got[0], rows[2]) and torch.equal(got[1], rows[1]) and torch.equal(got[2], rows[3])
    # refresh a resident id: updated in place, frequency grows, no new slot taken
    occupied = int((cache.ids >= 0).sum())
    cache.insert(torch.tensor([3]), torch.full((1, 4), -1.0))
    assert int((cache.ids >= 0).sum()) == occupied
    assert torch.equal(cache.lookup(torch.tensor([3]))[1][0], torch.full((4,), -1.0))
    # overflow: the least-frequently used slots are replaced, resident hot ids stay
    cache.insert(torch.arange(100, 106), torch.ones(6, 4))
    assert int((cache.ids >= 0).sum()) == 8
    assert bool(cache.lookup(torch.tensor([3]))[0][0])  # frequency 3 after two lookups and a refresh


def test_hot_cache_invariants_over_batches():
    """Over batches that overflow the cache: every id of the newest batch is
    resident with its newest row, every resident id holds the last row written
    for it, and the cache never holds more than its capacity."""
    cache = HotCache(capacity=16, dim=2)
    last_row = {}
    g = torch.Generator().manual_seed(3)
    for _ in range(6):
        ids = torch.randperm(40, generator=g)[:6]
        rows = torch.randn(6, 2, generator=g)
        cache.insert(ids, rows)
        last_row.update({int(v): rows[i] for i, v in enumerate(ids.tolist())})
        assert int((cache.ids >= 0).sum()) <= 16
        hit, got = cache.lookup(ids)
        assert bool(hit.all())
        assert torch.equal(got, rows)
    for v in cache.ids.tolist():
        if v >= 0:
            assert torch.equal(cache.lookup(torch.tensor([v]))[1][0], last_row[v])


def test_decay_cache_expires_old_versions():
    d = DecayCache(max_versions=2)
    for v in range(4):
        d.put(v, torch.tensor([v]), torch.zeros(1, 2))
    d.expire(3)
    assert sorted(d.entries) == [2, 3] and d.get(1) is None


def _ctdg_session(tmp_path):
    cfg = {"model": {"name": "tgn", "family": "tgn", "task": "temporal_link_prediction", "hidden_dim": 16},
           "data": {"root": str(tmp_path / "data"), "name": "ur_tgn", "format": "mock"},
           "train": {"epochs": 1, "batch_size": 16}, "runtime": {"device": "cpu"},
           "ctdg": {"dim_time": 8, "mailbox_slots": 1}}
    s = SchedulerSession.from_config(cfg)
    s.ctx.artifact_root = tmp_path / "art_tgn"
    s.prepare_data()
    s.build_runtime()
    return s


def _dtdg_session(tmp_path):
    cfg = {"model": {"name": "mpnn_lstm", "family": "mpnn_lstm", "task": "snapshot_node_regression",
                     "hidden_dim": 16},
           "data": {"root": str(tmp_path / "data"), "name": "ur_mpnn", "format": "mock"},
           "train": {"epochs": 1, "batch_size": 1, "snaps": 8}, "runtime": {"device": "cpu"},
           "graph": {"storage": "snapshots"}}
    s = SchedulerSession.from_config(cfg)
    s.ctx.artifact_root = tmp_path / "art_mpnn"
    s.prepare_data()
    s.build_runtime()
    return s


def test_ctdg_state_manager_and_runner(tmp_path):
    from starry_unigraph.runtime.state import CTDGStateManager

    s = _ctdg_session(tmp_path)
    results = run_units(s.build_runner(), "train", True)
    assert results and all("loss" in r for r in results)
    mb = s.ctdg_session.online_runtime.memory
    mgr = CTDGStateManager(mb, hot_capacity=32)
    ids = torch.arange(6)
    st = mgr.prepare(ids)
    assert torch.equal(st["memory"], mb.memory[ids]) and st["mailbox"].shape[0] == 6
    mgr.update({"memory_ids": ids[:2], "memory_rows": torch.ones(2, mb.hidden_dim),
                "memory_ts": torch.full((2,), 1e9)}, None)
    assert torch.equal(mb.memory[:2], torch.ones(2, mb.hidden_dim))
    mgr.patch(ids[2:4], torch.full((2, mb.hidden_dim), 3.0))
    mgr.step()
    assert mgr.describe()["version"] == 1 and mgr.describe()["hot"]["occupied"] == 2
    eng = s.build_pipeline_engine()
    assert type(eng.state_manager).__name__ == "CTDGStateManager"


def test_dtdg_runner_state_manager_and_plans(tmp_path):
    from starry_unigraph.runtime.state import DTDGStateManager

    s = _dtdg_session(tmp_path)
    runner = s.build_runner()
    results = run_units(runner, "train", True)
    assert results and len(runner.history) == len(results)
    mgr = DTDGStateManager()
    mgr.update({"state": (torch.ones(5, 3), torch.ones(5, 3))}, None)
    st = mgr.prepare(torch.arange(7))["state"]
    assert st[0].shape == (7, 3) and float(st[0][5:].abs().sum()) == 0.0
    blob = next(iter(s.snapshot_core.iter_train()))
    plan = StatePlan.from_window(blob)
    assert plan.describe()["writes"] == blob.current_graph.num_dst_nodes
    # single partition: no halo route, nothing to send
    assert SpatialPlan.from_route(getattr(blob.current_graph, "route", None)).volume() == 0


def test_spatial_plan_from_route():
    from starry_unigraph.backends.dtdg.runtime.route import Route

    r = Route(send_sizes=[0, 2, 1], recv_sizes=[3, 0, 2], send_index=torch.tensor([4, 7, 1]))
    plan = SpatialPlan.from_route(r)
    assert plan.volume() == 3 and plan.received() == 5
    assert plan.send_ids[1].tolist() == [4, 7] and plan.send_ids[2].tolist() == [1]
    assert plan.recv_ids[0].tolist() == [0, 1, 2] and plan.recv_ids[2].tolist() == [3, 4]


def test_route_volume_summary():
    from starry_unigraph.runtime.route.comm_plan import plan_from_routes

    class _Routes:
        send_sizes = [[1, 2], [0, 0], [4, 1]]
        recv_sizes = [[0, 3], [1, 0], [2, 2]]

    v = plan_from_routes(_Routes())
    assert v["send_rows"] == [3, 0, 5] and v["max_recv"] == 4 and v["total_send"] == 8


def test_store_memory_bank_and_state():
    """runtime.store: ring-slot mail writes per node, versioned updates, and a
    dense state view whose update / gather round-trip rows and mail."""
    import torch

    from starry_unigraph.runtime.store import MemoryBank, MemoryState, RNNState, TensorFeatureStore  # noqa: F401

    bank = MemoryBank(num_nodes=6, hidden_dim=2, edge_feat_dim=1, mailbox_slots=2)
    mails = torch.arange(4 * 5, dtype=torch.float32).view(4, 5)
    bank.write_mail(torch.tensor([3, 1, 3, 3]), mails, torch.tensor([1.0, 2.0, 3.0, 4.0]))
    # node 3 got three mails into two slots: slot 0 <- first, slot 1 <- second, slot 0 <- third
    assert torch.equal(bank.mailbox[3, 0], mails[3]) and torch.equal(bank.mailbox[3, 1], mails[2])
    assert torch.equal(bank.mailbox[1, 0], mails[1]) and int(bank.next_mail_pos[3]) == 1
    assert bank.mailbox_ts[3].tolist() == [4.0, 3.0]
    d = bank.describe()
    assert d["memory_version"] == 1 and d["num_local_nodes"] == 6 and d["mailbox_slots"] == 2
    st = MemoryState(6, 2, bank)
    st.update(torch.tensor([0, 5]), torch.tensor([[1.0, 2.0], [3.0, 4.0]]), mails=torch.ones(2, 5))
    rows, mb = st.gather(torch.tensor([5, 0]), mails=True)
    assert rows.tolist() == [[3.0, 4.0], [1.0, 2.0]] and torch.equal(mb[:, 0], torch.ones(2, 5))


def test_spatial_and_state_deps():
    import torch

    from starry_unigraph.runtime.route.comm_plan import SpatialDeps, StateDeps

    # 2 ranks x 3 clusters; send index grouped by cluster
    deps = SpatialDeps(torch.tensor([1, 2, 3, 4, 5, 6]), torch.tensor([6, 5, 4, 3, 2, 1]), torch.arange(10),
                       torch.tensor([0, 3, 7, 10]))
    r = deps.to_route([0, 2], num_clusters=3)
    assert r.send_sizes == [1 + 3, 4 + 6] and r.recv_sizes == [6 + 4, 3 + 1]
    assert r.send_index.tolist() == [0, 1, 2, 7, 8, 9]
    s = StateDeps(torch.tensor([1, 2]), torch.tensor([0, 1]), torch.tensor([5, 6, 7]),
                  [torch.tensor([0]), torch.tensor([1]), torch.tensor([0, 1])])
    f = s.stale_filter(torch.tensor([True, False, True]))
    assert f.write_notify.tolist() == [5, 7] and [t.tolist() for t in f.write_to_clusters] == [[0], [0, 1]]


def test_hot_cache_lookup_at_large_capacity():
    """A cache larger than a dense id-by-slot comparison would allow still hits."""
    cache = HotCache(capacity=200_000, dim=2)
    ids = torch.arange(0, 300_000, 2)
    cache.insert(ids, torch.stack([ids.float(), -ids.float()], 1))
    hit, got = cache.lookup(torch.tensor([4, 5, 299_998, 7]))
    assert hit.tolist() == [True, False, True, False]
    assert got[0].tolist() == [4.0, -4.0] and got[2].tolist() == [299_998.0, -299_998.0]
    assert got[1].tolist() == [0.0, 0.0]
    assert cache.describe()["hits"] == 2 and cache.describe()["misses"] == 2


def test_backend_adapters_expose_every_mode_as_chunks(tmp_path):
    """CTDG batches, Flare windows and chunk-mode chunks all come out of their
    GraphBackend as ChunkAtomic units whose events and T-CSR rows are the
    runtime's own (reference tests/test_orthogonal_separation.py::test_backend_adapters)."""
    from starry_unigraph.runtime.backend_adapters import CTDGGraphBackend, ChunkGraphBackend, FlareGraphBackend
    from test_session import _session

    s = _session(tmp_path / "c", family="tgn")
    s.prepare_data()
    s.build_runtime()
    rt = s.ctdg_session.online_runtime
    back = CTDGGraphBackend(s.ctdg_session)
    chunks = list(back.iter_batches("train", 8))
    batches = list(rt.iter_batches("train", 8))
    assert len(chunks) == len(batches) and back.describe()["backend"] == "ctdg_online"
    csr = rt.sampler.csr("train")
    for ch, b in zip(chunks, batches):
        assert torch.equal(ch.events["src"], b.src) and torch.equal(ch.events["eid"], b.event_ids)
        for i, v in enumerate(ch.node_set.tolist()):
            a, e = int(ch.tcsr_rowptr[i]), int(ch.tcsr_rowptr[i + 1])
            lo, hi = int(csr.rowptr[v]), int(csr.rowptr[v + 1])
            assert torch.equal(ch.tcsr_edge_id[a:e], csr.eid[lo:hi].cpu())
    d = _session(tmp_path / "d", family="mpnn_lstm")
    d.prepare_data()
    d.build_runtime()
    windows = list(FlareGraphBackend(d.snapshot_core).iter_batches("train", 1))
    assert windows and all(w.events["graph"].num_edges() > 0 for w in windows)
    assert all(w.num_events == w.events["graph"].num_edges() for w in windows)
    from test_components import _chunk_session

    k = _chunk_session(tmp_path / "k")
    k.prepare_data()
    k.build_runtime()
    units = list(ChunkGraphBackend(k.snapshot_core).iter_batches("train", 1))
    assert [u.chunk_id for u in units] == [c.chunk_id for c in k.snapshot_core.iter_chunks("train")]


def test_predict_result_has_one_shape_in_every_mode(tmp_path):
    """predict() returns PredictionResult(predictions: list of floats, targets, meta with
    split and graph_mode) in CTDG, DTDG and chunk mode alike."""
    from starry_unigraph.types import PredictionResult
    from test_components import _chunk_session
    from test_session import _session

    sessions = {"ctdg": _session(tmp_path / "c", family="tgn"), "dtdg": _session(tmp_path / "d", family="tgcn"),
                "chunk": _chunk_session(tmp_path / "k")}
    for mode, s in sessions.items():
        s.prepare_data()
        s.build_runtime()
        r = s.predict("test")
        assert isinstance(r, PredictionResult) and r.predictions
        assert all(isinstance(x, float) for x in r.predictions)
        assert r.meta["split"] == "test" and r.meta["graph_mode"] in ("ctdg", "dtdg")
        assert r.targets is None or len(r.targets) == len(r.predictions)


def test_missing_route_manifest_fails_early(tmp_path):
    from test_session import _session

    s = _session(tmp_path, family="mpnn_lstm")
    s.prepare_data()
    (s.ctx.artifact_root / "routes" / "manifest.json").unlink()
    s.prepared = None
    with pytest.raises(FileNotFoundError, match="route"):
        s.build_runtime()


@pytest.mark.parametrize("mode", ["ctdg", "dtdg", "chunk"])
def test_pipeline_engine_trains_like_the_session(tmp_path, mode):
    """The unified engine over a session's own runtime trains: an engine epoch gives the
    same losses as the session's run_epoch on a twin session, and moves the parameters
    (reference architecture: PipelineEngine x GraphBackend x TaskAdapter x StateManager)."""
    from test_components import _chunk_session
    from test_session import _session

    def make(sub):
        s = _chunk_session(tmp_path / sub) if mode == "chunk" else \
            _session(tmp_path / sub, family="tgn" if mode == "ctdg" else "mpnn_lstm")
        s.prepare_data()
        s.build_runtime()
        return s

    a, b = make("a"), make("b")
    before = [p.detach().clone() for p in b.runtime.model.parameters()]
    torch.manual_seed(1)  # dropout draws from the global stream: same start for both epochs
    ref = a.run_epoch("train")
    eng = b.build_pipeline_engine()
    torch.manual_seed(1)
    out = eng.run_epoch("train", batch_size=int(b.ctx.config["train"]["batch_size"]))
    ref_losses = [float(o["loss"]) for o in ref["outputs"] if o.get("meta", {}).get("batch_size", 1) != 0]
    got = out["losses"]
    assert got == pytest.approx(ref_losses, rel=1e-5) and len(got) > 0
    assert any(not torch.equal(x, y) for x, y in zip(before, b.runtime.model.parameters()))
    val = eng.run_epoch("val", batch_size=int(b.ctx.config["train"]["batch_size"]))
    assert val["num_batches"] > 0 and val["loss"] > 0
