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


@pytest.mark.parametrize("H,IN", [(64, 64), (32, 40), (128, 128)])
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
