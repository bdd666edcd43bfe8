"""Host C++ natives: T-CSR + sampler (against the vectorised torch oracle), time split,
partitioner, TPPR, utilities."""
import pytest
import torch

N = pytest.importorskip("starry_unigraph._native")


def _stream(n_nodes=200, m=5000, seed=0):
    g = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n_nodes, (m,), generator=g)
    dst = torch.randint(0, n_nodes, (m,), generator=g)
    ts = torch.sort(torch.randint(0, 100000, (m,), generator=g)).values
    return src, dst, ts


def test_recent_sampler_matches_torch_oracle():
    from starry_unigraph.backends.ctdg.runtime.sampler import TemporalCSR

    src, dst, ts = _stream()
    eid = torch.arange(src.numel())
    tnb = N.get_neighbors("test_recent", src, dst, 200, 0, eid, None, None, ts)
    s = N.ParallelSampler(tnb, 200, src.numel(), 4, [7], 1, "recent", -1, torch.zeros(1, dtype=torch.int32),
                          torch.zeros(1, dtype=torch.int32), 1.0)
    roots = torch.arange(0, 200, 3)
    rts = torch.full((roots.numel(),), 60000, dtype=torch.int64)
    s.neighbor_sample_from_nodes(roots, rts)
    blk = s.get_ret()[0]
    csr = TemporalCSR.build(src, dst, eid, ts, 200)
    ref = csr.sample_torch(roots, rts, 7, "recent")
    m = ref.mask()
    assert torch.equal(blk.sample_nodes(), ref.nbr[m])
    assert torch.equal(blk.eid(), ref.eid[m])
    assert torch.equal(blk.delta_ts(), ref.dt[m].long())
    assert torch.equal(blk.src_index(), torch.arange(roots.numel()).repeat_interleave(ref.count.long()))


def test_uniform_sampler_distribution():
    src = torch.arange(10).repeat(100)                 # node 0 receives from 10 sources uniformly
    dst = torch.zeros(1000, dtype=torch.long)
    ts = torch.arange(1000)
    tnb = N.get_neighbors("test_uniform", src, dst, 10, 0, torch.arange(1000), None, None, ts)
    s = N.ParallelSampler(tnb, 10, 1000, 2, [50], 1, "uniform", -1, torch.zeros(1, dtype=torch.int32),
                          torch.zeros(1, dtype=torch.int32), 1.0)
    counts = torch.zeros(10)
    for _ in range(40):
        s.neighbor_sample_from_nodes(torch.zeros(1, dtype=torch.long), torch.tensor([1000]))
        counts += torch.bincount(s.get_ret()[0].sample_nodes(), minlength=10).float()
    expected = counts.sum() / 10
    chi2 = float(((counts - expected) ** 2 / expected).sum())
    assert chi2 < 30.0  # 9 dof, p ~ 5e-4


def test_multilayer_and_boundary_policies():
    src, dst, ts = _stream()
    eid = torch.arange(src.numel())
    tnb = N.get_neighbors("test_ml", src, dst, 200, 0, eid, None, None, ts)
    for pol in ["boundery_recent_uniform", "boundery_recent_decay"]:
        s = N.ParallelSampler(tnb, 200, src.numel(), 2, [5, 3], 2, pol, 0,
                              (eid % 2).to(torch.int32), (torch.arange(200) % 2).to(torch.int32), 0.5)
        s.neighbor_sample_from_nodes(torch.arange(50), torch.full((50,), 80000))
        r = s.get_ret()
        assert len(r) == 2
        assert r[0].sample_nodes().numel() <= 50 * 6


def test_tnb_pickle_and_updates():
    import pickle

    src, dst, ts = _stream(50, 500)
    tnb = N.get_neighbors("test_pickle", src, dst, 50, 0, torch.arange(500), None, torch.ones(500), ts)
    t2 = pickle.loads(pickle.dumps(tnb))
    assert t2.neighbors == tnb.neighbors and t2.timestamp == tnb.timestamp
    t2.update_neighbors_with_time(torch.tensor([1]), torch.tensor([2]), torch.tensor([200000]),
                                  torch.tensor([500]), 0, None)
    assert t2.deg[2] == tnb.deg[2] + 1


def test_time_split_groups_are_contiguous():
    src, dst, ts = _stream(100, 3000)
    r = N.adaptive_split(src, dst, ts.double(), 200, 0.5)
    g = r.group_index
    assert g.numel() == 3000 and int(g[0]) == 0
    assert bool((g[1:] - g[:-1] >= 0).all()) and bool((g[1:] - g[:-1] <= 1).all())
    d = N.adaptive_split(src, dst, ts.double(), 200, 0.5, enable_drop=True, drop_rate=0.5)
    assert 0.0 <= d.drop_proportion <= 0.6


def test_partitioner_balanced_and_better_than_random():
    g = torch.Generator().manual_seed(0)
    # 4 dense communities + sparse inter-community edges
    comm = torch.arange(2000) % 4
    src = torch.randint(0, 2000, (30000,), generator=g)
    same = torch.rand(30000, generator=g) < 0.9
    dst = torch.where(same, (torch.randint(0, 500, (30000,), generator=g) * 4 + comm[src]), torch.randint(0, 2000, (30000,), generator=g))
    p = N.partition_graph(src, dst, 2000, 4, 1.05, 5, 0)
    sizes = torch.bincount(p, minlength=4)
    assert int(sizes.max()) <= int(1.06 * 500) + 1
    cut = float((p[src] != p[dst]).float().mean())
    rnd = torch.randint(0, 4, (2000,), generator=g)
    assert cut < float((rnd[src] != rnd[dst]).float().mean())


def test_partitioner_weighted_balance_on_power_law_graph():
    """Vertex weight (1 - s) / N + s * degree / D: on a power-law graph node
    balance alone leaves one part with most edge endpoints; the weighted balance
    keeps every part's weight within the imbalance bound (a single vertex may
    exceed it)."""
    g = torch.Generator().manual_seed(1)
    n, m, k = 20000, 200000, 4
    w = torch.arange(1, n + 1, dtype=torch.float64) ** (-1 / 1.1)
    src = torch.multinomial(w, m, replacement=True, generator=g)
    dst = torch.multinomial(w, m, replacement=True, generator=g)
    keep = src != dst
    src, dst = src[keep], dst[keep]
    deg = (torch.bincount(src, minlength=n) + torch.bincount(dst, minlength=n)).double()
    share = 0.3
    vw = (1 - share) / n + share * deg / deg.sum()
    for s, bound in ((0.0, None), (share, 1.03)):
        p = N.partition_graph(src, dst, n, k, 1.03, 3, 0, s)
        weight = torch.zeros(k, dtype=torch.float64).index_add_(0, p, vw)
        ratio = float(weight.max() / weight.mean())
        if bound is None:
            node_only = ratio
        else:
            assert ratio <= bound + float(vw.max() / weight.mean()), ratio
            assert ratio < node_only


def test_tppr_streaming_and_pruned():
    src, dst, ts = _stream(30, 300)
    eid = torch.arange(300)
    tnb = N.get_neighbors("test_tppr", src, dst, 30, 0, eid, None, None, ts)
    comp = N.ParallelTppRComputer(tnb, 30, 300, 2, 5, 2, 1, [0.1], [0.9])
    fake = torch.randint(0, 30, (100,))
    comp.streaming_topk(torch.cat([src[:100], dst[:100], fake]), ts[:100], eid[:100])
    ret = comp.get_ret()[0]
    assert len(ret) == 300
    assert all(b.sample_nodes().numel() <= 5 for b in ret)
    comp.get_pruned_topk(torch.arange(10), torch.full((10,), 100000), 0)
    assert len(comp.get_ret()[0]) == 10


def test_utils():
    assert N.heads_unique(torch.tensor([3, 1, 3, 2]), torch.tensor([2, 5]), 1).tolist() == [2, 5, 3, 1]
    parts = N.divide_nodes_to_part(torch.tensor([0, 5, 9, 3]), [0, 4, 8, 12], 1)
    assert [p.tolist() for p in parts] == [[0, 3], [5], [9]]
    assert N.sparse_get_index(torch.tensor([7, 8, 9]), torch.tensor([9, 7])).tolist() == [1, -1, 0]
    m, s = N.get_norm_temporal(torch.tensor([0, 0, 0]), torch.tensor([1, 1, 1]), torch.tensor([0.0, 2.0, 4.0]), 2)
    assert abs(m - 2.0) < 1e-9 and abs(s) < 1e-9


def _policy_dataset(n_nodes=30, n_events=600, seed=4):
    from types import SimpleNamespace

    g = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n_nodes, (n_events,), generator=g)
    dst = torch.randint(0, n_nodes, (n_events,), generator=g)
    ts = torch.sort(torch.randint(0, 10_000, (n_events,), generator=g)).values
    weight = (torch.arange(n_events) % 2).float() * torch.rand(n_events, generator=g)  # odd events only
    graph = {"row": src, "col": dst, "eid": torch.arange(n_events), "ts": ts, "weight": weight}
    return SimpleNamespace(num_nodes=n_nodes, num_edges=n_events, src=src, node_parts=None, edge_parts=None,
                           partition_rank=0, sampler_graph=lambda split: graph)


def test_session_sampler_native_layout_matches_vectorised():
    """The host sampler's flat blocks, laid out as [roots, k], equal the vectorised
    recent sampler over two layers."""
    from starry_unigraph.backends.ctdg.runtime.sampler import NativeTemporalSampler

    ds = _policy_dataset()
    s = NativeTemporalSampler(ds, fanout=[4, 3], history=2, strategy="recent")
    roots, rts = torch.arange(30), torch.full((30,), 6000)
    a, b = s.sample("train", roots, rts), s._sample_native("train", roots, rts)
    for x, y in zip(a.blocks, b.blocks):
        m = x.mask()
        assert torch.equal(x.count.long(), y.count.long())
        assert torch.equal(x.nbr[m], y.nbr[m]) and torch.equal(x.eid[m], y.eid[m]) and torch.equal(x.dt[m], y.dt[m])


def test_session_sampler_weighted_and_boundary_policies():
    from starry_unigraph.backends.ctdg.runtime.sampler import NativeTemporalSampler

    ds = _policy_dataset()
    roots, rts = torch.arange(30), torch.full((30,), 9000)
    w = NativeTemporalSampler(ds, fanout=[8], history=1, strategy="weighted").sample("train", roots, rts).blocks[0]
    picked = w.eid[w.mask()]
    assert picked.numel() > 0 and bool((picked % 2 == 1).all())  # zero-weight events are never drawn
    # boundary policy: with keep probability 0 no candidate owned by the other rank survives
    ds.node_parts = torch.arange(30) % 2
    ds.edge_parts = ds.node_parts[ds.src]
    blk = NativeTemporalSampler(ds, fanout=[6], history=1, strategy="boundery_recent_uniform",
                                boundary_p=0.0).sample("train", roots, rts).blocks[0]
    m = blk.mask()
    assert blk.nbr[m].numel() > 0
    assert bool((ds.node_parts[blk.nbr[m]] == 0).all()) and bool((ds.edge_parts[blk.eid[m]] == 0).all())
    # keep probability 1: the boundary policy takes the most recent candidates (newest first)
    full = NativeTemporalSampler(ds, fanout=[6], history=1, strategy="boundery_recent_uniform",
                                 boundary_p=1.0).sample("train", roots, rts).blocks[0]
    rec = NativeTemporalSampler(ds, fanout=[6], history=1, strategy="recent").sample("train", roots, rts).blocks[0]
    assert torch.equal(full.count, rec.count)
    for i in range(roots.numel()):
        n = int(rec.count[i])
        assert sorted(full.eid[i, :n].tolist()) == sorted(rec.eid[i, :n].tolist())
    with pytest.raises(ValueError):
        NativeTemporalSampler(ds, fanout=[6], history=1, strategy="nearest")


def test_session_trains_with_weighted_sampling_and_cuda_guard(tmp_path, monkeypatch):
    from starry_unigraph import SchedulerSession

    cfg = {"model": {"name": "tgn", "family": "tgn", "task": "temporal_link_prediction", "hidden_dim": 16},
           "data": {"root": str(tmp_path / "d"), "name": "w", "format": "synthetic",
                    "synthetic": {"preset": "tgn_cpu", "num_events": 1500}},
           "train": {"epochs": 1, "batch_size": 100}, "runtime": {"device": "cpu"},
           "ctdg": {"dim_time": 8, "mailbox_slots": 1}, "sampling": {"strategy": "weighted"}}
    s = SchedulerSession.from_config(cfg)
    s.ctx.artifact_root = tmp_path / "art"
    s.prepare_data()
    s.build_runtime()
    assert s.run_epoch("train")["loss"] > 0
    # the CUDA step samples recent / uniform only: other policies are refused there, not run as uniform
    from starry_unigraph.backends.ctdg.runtime.factory import build_ctdg_runtime

    monkeypatch.setattr(torch.cuda, "is_available", lambda: True)
    s.ctx.config["runtime"]["device"] = "cuda"
    with pytest.raises(ValueError, match="host sampler"):
        build_ctdg_runtime(s.ctx)
