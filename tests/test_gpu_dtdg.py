"""DTDG sm_100a kernels (CSR SpMM, fused LSTM cell, tcgen05 linear autograd) and
the Flare models on CUDA against the PyTorch CPU path."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return float((a - b).norm() / (b.norm() + 1e-12))


def _block(n_dst=300, n_halo=50, m=3000, seed=0):
    from starry_unigraph.data.partition import SnapshotBlock

    g = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n_dst + n_halo, (m,), generator=g)
    dst = torch.randint(0, n_dst, (m,), generator=g)
    b = SnapshotBlock(num_src_nodes=n_dst + n_halo, num_dst_nodes=n_dst, edge_src=src, edge_dst=dst)
    b.edata["gcn_norm"] = torch.rand(m, generator=g)
    return b


@pytest.mark.parametrize("F", [16, 64, 128, 40])
def test_spmm_fwd_bwd(F):
    from starry_unigraph.data.partition import SnapshotBlock
    from starry_unigraph.ops.dtdg import gcn_aggregate

    b = _block()
    x = torch.randn(b.num_src_nodes, F, requires_grad=True)
    ref = gcn_aggregate(b, x)
    ref.backward(torch.ones_like(ref))
    bc = SnapshotBlock(b.num_src_nodes, b.num_dst_nodes, b.edge_src.cuda(), b.edge_dst.cuda(),
                       edata={"gcn_norm": b.edata["gcn_norm"].cuda()})
    xc = x.detach().cuda().requires_grad_()
    out = gcn_aggregate(bc, xc)
    out.backward(torch.ones_like(out))
    assert _rel(out.cpu(), ref.detach()) < 1e-5
    assert _rel(xc.grad.cpu(), x.grad) < 1e-5


@pytest.mark.parametrize("F", [64, 128, 100])
def test_spmm_csr_skewed_rows(F):
    """Rows of every kind the edge-chunk walk meets: hubs spanning several chunks,
    runs of empty rows longer than the 32-row look-ahead window, single-edge rows;
    plain and accumulating output, against an fp64 index_add reference."""
    import starry_unigraph._C as C

    g = torch.Generator().manual_seed(7)
    n_rows, n_src = 6000, 4000
    deg = torch.randint(0, 4, (n_rows,), generator=g)
    deg[100] = 5000           # hub: about twenty 256-edge chunks
    deg[2000] = 700
    deg[3000:3100] = 0        # 100 empty rows in a row
    deg[4000:4300] = 1
    rowptr = torch.zeros(n_rows + 1, dtype=torch.long)
    rowptr[1:] = deg.cumsum(0)
    nnz = int(rowptr[-1])
    col = torch.randint(0, n_src, (nnz,), generator=g, dtype=torch.int32)
    val = torch.rand(nnz, generator=g)
    x = torch.randn(n_src, F, generator=g)
    row_of = torch.repeat_interleave(torch.arange(n_rows), deg)
    ref = torch.zeros(n_rows, F, dtype=torch.float64).index_add_(
        0, row_of, val.double()[:, None] * x.double()[col.long()])
    dev = lambda t: t.cuda()  # noqa: E731
    out = C.spmm_csr(dev(rowptr), dev(col), dev(val), dev(x), n_rows, None, False)
    assert _rel(out.cpu().double(), ref) < 1e-6
    base = torch.randn(n_rows, F, generator=g)
    acc = dev(base.clone())
    C.spmm_csr(dev(rowptr), dev(col), dev(val), dev(x), n_rows, acc, True)
    assert _rel(acc.cpu().double(), ref + base.double()) < 1e-6
    # item plan (64 features): hubs split over items with atomic adds, empty rows as zero items;
    # the output starts from garbage to show every row is written
    from starry_unigraph.data.partition import spmm_plan

    for max_edges, warps in ((128, None), (16, 37)):
        plan = spmm_plan(dev(rowptr), max_edges, warps)
        out = torch.full((n_rows, F), float("nan"), device="cuda")
        C.spmm_csr(dev(rowptr), dev(col), dev(val), dev(x), n_rows, out, False, plan)
        assert _rel(out.cpu().double(), ref) < 1e-6, (max_edges, warps)


@pytest.mark.parametrize("H,FX,strided", [(64, 64, True), (128, 128, True), (32, 20, False)])
def test_rgru_cell_fused(H, FX, strided):
    """Reset-gated GRU cell (T-GCN gates / MatGRU) on the tcgen05 path against
    the fp32 torch math: outputs and every gradient."""
    from starry_unigraph.ops.dtdg import rgru_cell

    torch.manual_seed(0)
    rows = 700
    if strided:  # gate inputs as column chunks of one [rows, 3 FX] tensor (T-GCN's urc)
        urc = torch.randn(rows, 3 * FX)
    else:
        urc = torch.randn(rows, FX)
    h0 = torch.randn(rows, H)
    ws = [torch.randn(H, FX + H) * 0.2 for _ in range(3)]
    bs = [torch.randn(H) * 0.1 for _ in range(3)]

    def run(dev):
        u = urc.detach().to(dev).clone().requires_grad_()
        h = h0.detach().to(dev).clone().requires_grad_()
        w = [t.detach().to(dev).clone().requires_grad_() for t in ws]
        b = [t.detach().to(dev).clone().requires_grad_() for t in bs]
        xz, xr, xc = u.chunk(3, -1) if strided else (u, u, u)
        out = rgru_cell(xz, xr, xc, h, w[0], b[0], w[1], b[1], w[2], b[2])
        (out * torch.linspace(-1, 1, H, device=dev)).sum().backward()
        return [out] + [t.grad for t in (u, h, *w, *b)]

    ref = run("cpu")
    got = run("cuda")
    for a, r in zip(got, ref):
        assert _rel(a.detach().cpu(), r.detach()) < 1.5e-2


@pytest.mark.parametrize("H,IN", [(64, 64), (32, 40), (128, 128), (20, 12)])
def test_lstm_cell_fused(H, IN):
    from starry_unigraph.runtime.modules.rnn_cells import _LSTMCell

    torch.manual_seed(0)
    cell = _LSTMCell(IN, H)
    x = torch.randn(500, IN)
    h0, c0 = torch.randn(500, H), torch.randn(500, H)
    hr, cr = cell(x, (h0, c0))
    (hr.sum() + cr.pow(2).sum()).backward()
    gref = [p.grad.clone() for p in cell.parameters()]
    cc = _LSTMCell(IN, H).cuda()
    cc.load_state_dict(cell.state_dict())
    xg = x.cuda().requires_grad_()
    hg, cg = cc(xg, (h0.cuda(), c0.cuda()))
    (hg.sum() + cg.pow(2).sum()).backward()
    assert _rel(hg.cpu(), hr.detach()) < 1.5e-2
    assert _rel(cg.cpu(), cr.detach()) < 1.5e-2
    for a, b in zip(cc.parameters(), gref):
        assert _rel(a.grad.cpu(), b) < 3e-2


def test_lstm_cell_no_state():
    from starry_unigraph.runtime.modules.rnn_cells import _LSTMCell

    cell = _LSTMCell(64, 64)
    x = torch.randn(200, 64)
    hr, cr = cell(x, None)
    cc = _LSTMCell(64, 64).cuda()
    cc.load_state_dict(cell.state_dict())
    hg, cg = cc(x.cuda(), None)
    assert _rel(hg.cpu(), hr.detach()) < 1.5e-2


@pytest.mark.parametrize("family", ["mpnn_lstm", "tgcn", "evolvegcn"])
def test_flare_model_cuda_matches_cpu(tmp_path, family):
    from starry_unigraph import SchedulerSession

    losses = {}
    for dev in ("cpu", "cuda"):
        cfg = {"model": {"name": family, "family": family, "task": "snapshot_node_regression", "hidden_dim": 32},
               "data": {"root": "./data", "name": "gdt", "format": "synthetic",
                        "synthetic": {"num_nodes": 2000, "num_snapshots": 8, "edges_per_snapshot": 20000,
                                      "churn": 0.3, "feat_dim": 16}},
               "train": {"epochs": 1, "batch_size": 1, "lr": 0.0}, "runtime": {"device": dev},
               "graph": {"storage": "snapshots"}, "dtdg": {"chunk_order": None, "chunk_decay": None}}
        s = SchedulerSession.from_config(cfg)
        s.ctx.artifact_root = tmp_path / dev
        s.prepare_data()
        s.build_runtime()
        losses[dev] = s.run_epoch("train")["loss"]
    assert abs(losses["cpu"] - losses["cuda"]) <= 2e-2 * abs(losses["cpu"]) + 1e-4, losses


@pytest.mark.parametrize("family", ["mpnn_lstm", "tgcn"])
def test_graph_replayed_steps_match_eager(tmp_path, family):
    """Training windows run as captured CUDA graphs (forward, backward, Adam) give
    the losses and parameters of eager steps, including windows replayed a second
    time (second epoch over the same windows)."""
    from starry_unigraph import SchedulerSession
    from starry_unigraph.backends.dtdg.runtime.training import run_flare_train_step

    results = {}
    for graphs in (False, True):
        cfg = {"model": {"name": family, "family": family, "task": "snapshot_node_regression", "hidden_dim": 32,
                         "window": {"size": 3}},
               "data": {"root": "./data", "name": "gdt", "format": "synthetic",
                        "synthetic": {"num_nodes": 3000, "num_snapshots": 10, "edges_per_snapshot": 30000,
                                      "churn": 0.3, "feat_dim": 16}},
               "train": {"epochs": 1, "batch_size": 1, "lr": 1e-3},
               "runtime": {"device": "cuda", "cuda_graphs": graphs},
               "graph": {"storage": "snapshots"},
               "dtdg": {"chunk_order": None, "chunk_decay": None, "window_from_size": True}}
        s = SchedulerSession.from_config(cfg)
        s.ctx.artifact_root = tmp_path / f"g{int(graphs)}"
        s.prepare_data()
        s.build_runtime()
        blobs = list(s.snapshot_core.iter_train())
        assert len(blobs) >= 4
        losses = [float(run_flare_train_step(s.runtime, b, {"meta": {}}, need_host=False)["loss"])
                  for b in blobs + blobs]  # every window twice: captures, then replays
        torch.cuda.synchronize()
        sg = s.runtime.state.get("step_graphs")
        if graphs:
            assert sg is not None and sg.captures == len(blobs)  # the two eager warm-up windows on the 2nd pass
        results[graphs] = (losses, [p.detach().cpu().clone() for p in s.runtime.model.parameters()])
    (le, pe), (lg, pg) = results[False], results[True]
    torch.testing.assert_close(torch.tensor(lg), torch.tensor(le), rtol=1e-3, atol=1e-5)
    # weight-gradient atomics sum in a run-dependent order; Adam turns last-bit differences of
    # near-zero gradients into differences of up to lr in single elements
    for a, b in zip(pg, pe):
        torch.testing.assert_close(a, b, rtol=1e-2, atol=2e-4)
