"""Fused sm_100a TGN step against the PyTorch CPU path of the same runtime
(reference semantics), with dropout disabled so both are deterministic."""
import copy

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg(device, **over):
    cfg = {"model": {"name": "tgn", "family": "tgn", "task": "temporal_link_prediction", "hidden_dim": 32},
           "data": {"root": "./data", "name": "gputest", "format": "synthetic",
                    "synthetic": {"preset": "tgn_cpu", "num_events": 4000, "edge_dim": 8, "num_src": 300,
                                  "num_dst": 100}},
           "train": {"epochs": 1, "batch_size": 100, "lr": 1e-3},
           "runtime": {"device": device, "cuda_graphs": False},
           "ctdg": {"mailbox_slots": 1, "dim_time": 16, "num_head": 2, "dropout": 0.0, "att_dropout": 0.0},
           "sampling": {"neighbor_limit": [5], "strategy": "recent", "history": 1}}
    for k, v in over.items():
        cfg[k].update(v)
    return cfg


def _session(device, tmp_path, **over):
    from starry_unigraph import SchedulerSession

    s = SchedulerSession.from_config(_cfg(device, **over))
    s.ctx.artifact_root = tmp_path / device.replace(":", "_")
    s.prepare_data()
    s.build_runtime()
    return s


def test_sampler_kernel_matches_torch(tmp_path):
    from starry_unigraph.ops import cuda_ext

    C = cuda_ext()
    s = _session("cuda", tmp_path)
    rt = s.ctdg_session.online_runtime
    csr = rt.sampler.csr("train")
    R = 64
    roots = torch.randperm(rt.dataset.num_nodes, device="cuda")[:R]
    rts = torch.tensor([int(rt.dataset.ts[1500])], device="cuda", dtype=torch.int64)
    ref = csr.sample_torch(roots, rts.expand(R), 5, "recent")
    k = 5
    out_nbr = torch.zeros(R * k, dtype=torch.int64, device="cuda")
    out_eid = torch.zeros_like(out_nbr)
    out_dt = torch.zeros(R * k, device="cuda")
    out_cnt = torch.zeros(R, dtype=torch.int32, device="cuda")
    tot = torch.zeros(1, dtype=torch.int32, device="cuda")
    n_roots = torch.tensor([R], dtype=torch.int32, device="cuda")
    step = torch.zeros(1, dtype=torch.int64, device="cuda")
    C.tgn_sample(roots, n_roots, rts, csr.rowptr, csr.nbr, csr.eid, csr.ts, k, 0, 0, step, out_nbr, out_eid, out_dt,
                 out_cnt, tot)
    torch.cuda.synchronize()
    assert torch.equal(out_cnt.long().cpu(), ref.count.long().cpu())
    assert torch.equal(out_nbr.view(R, k).cpu(), ref.nbr.cpu())
    assert torch.equal(out_eid.view(R, k).cpu(), ref.eid.cpu())
    assert torch.allclose(out_dt.view(R, k).cpu(), ref.dt.cpu())
    assert int(tot) == int(ref.count.sum())


# tolerances of the fused step against the fp32 CPU oracle per operand precision
# (gradient errors of both are dominated by the time encoding of large time deltas: fp32 w * dt
# has an ulp of ~0.25 rad at dt ~ 1e6, so cos / sin there differ between any two implementations)
TOL = {"bf16": {"loss": 1e-2, "pred": 1e-2, "table": 2e-2, "grad": 5e-2},
       "tf32": {"loss": 3e-3, "pred": 3e-3, "table": 5e-3, "grad": 5e-2}}


@pytest.mark.parametrize("precision", ["tf32", "bf16"])
@pytest.mark.parametrize("slots", [1, 2])
def test_fused_forward_and_memory_match_cpu_oracle(tmp_path, slots, precision):
    """lr = 0: parameters stay fixed, so per-step losses, the memory table and the
    mailbox isolate the forward pass and the memory/mailbox semantics."""
    tol = TOL[precision]
    g = _session("cuda", tmp_path, ctdg={"mailbox_slots": slots}, train={"lr": 0.0},
                 runtime={"precision": precision})
    c = _session("cpu", tmp_path, ctdg={"mailbox_slots": slots}, train={"lr": 0.0})
    rg, rc = g.ctdg_session.online_runtime, c.ctdg_session.online_runtime
    for a, b in zip(rg.model.state_dict().values(), rc.model.state_dict().values()):
        assert torch.allclose(a.cpu(), b)
    eng = rg.engine
    for i, batch in enumerate(list(rc.iter_batches("train", 100))[:8]):
        res_g = rg.train_step(batch)
        neg = eng.neg[: batch.size].cpu()
        rc._negative_sample = lambda b, neg=neg: neg
        res_c = rc.train_step(batch)
        lg, lc = res_g["loss"], res_c["loss"]
        assert abs(lg - lc) <= tol["loss"] * max(1.0, abs(lc)), (i, lg, lc)
        pg, pc = torch.tensor(res_g["predictions"]), torch.tensor(res_c["predictions"])
        assert float((pg - pc).abs().max()) < tol["pred"], (i, float((pg - pc).abs().max()))
    from starry_unigraph.ops import check_status

    check_status()
    mg, mc = rg.memory, rc.memory
    assert torch.allclose(mg.memory.cpu(), mc.memory, atol=tol["table"], rtol=tol["table"])
    assert torch.allclose(mg.mailbox.cpu(), mc.mailbox, atol=tol["table"], rtol=tol["table"])
    assert torch.equal(mg.next_mail_pos.cpu(), mc.next_mail_pos)


@pytest.mark.parametrize("precision", ["tf32", "bf16"])
def test_fused_gradients_match_autograd(tmp_path, precision):
    """Gradients of every trainable parameter after the same steps (lr = 0 keeps
    both models identical; gradients of the last step are compared)."""
    g = _session("cuda", tmp_path, train={"lr": 0.0}, runtime={"precision": precision})
    c = _session("cpu", tmp_path, train={"lr": 0.0})
    rg, rc = g.ctdg_session.online_runtime, c.ctdg_session.online_runtime
    eng = rg.engine
    conv = rc.model.conv
    rec = {}

    def keep(name, flat_to=None):
        def hook(mod, inp, out):
            if name == "t":
                rec.setdefault("t", []).append(inp[0].detach().reshape(-1))
            out.register_hook(lambda gr: rec.setdefault(name, []).append(gr.detach().reshape(-1, gr.shape[-1])))
        return hook

    conv.time_enc.register_forward_hook(keep("t"))
    conv.w_k.register_forward_hook(keep("dK"))
    conv.w_v.register_forward_hook(keep("dV"))
    for batch in list(rc.iter_batches("train", 100))[:5]:
        rg.train_step(batch)
        neg = eng.neg[: batch.size].cpu()
        rc._negative_sample = lambda b, neg=neg: neg
        rec.clear()
        rc.train_step(batch)
    max_dt = float(rc.dataset.ts.max())
    # the time-encoder weight gradient is sum_e d cos(w dt_e + b)/dw * (dK_e W_k[:, time] + dV_e W_v[:, time]);
    # its terms cancel, so its error is judged against the sum of the terms' magnitudes, with the upstream
    # products taken in absolute value (errors of dK/dV from bf16 operands propagate at that scale)
    T = conv.time_enc.w.weight.shape[0]
    w64 = conv.time_enc.w.weight.detach().view(-1).double()
    b64 = conv.time_enc.w.bias.detach().view(-1).double()
    t = [x for x in rec["t"] if x.numel() == rec["dK"][0].shape[0]][0].double()
    wk, wv = conv.w_k.weight.detach()[:, -T:].abs(), conv.w_v.weight.detach()[:, -T:].abs()
    up = (rec["dK"][0].abs() @ wk + rec["dV"][0].abs() @ wv).double()
    scale = (torch.sin(t[:, None] * w64 + b64).abs() * t.abs()[:, None] * up).sum(0)
    errs = {}
    for (n, pg), pc in zip(rg.model.named_parameters(), rc.model.parameters()):
        a, b = pg.grad.detach().cpu(), pc.grad.detach()
        if n == "conv.w_k.bias":
            # exact gradient is zero: the softmax over a root's edges is invariant to the shift q . b_k,
            # which is the same for every edge; both sides hold rounding residue only
            errs[n] = float(a.norm() / (dict(rg.model.named_parameters())["conv.w_k.weight"].grad.norm().cpu()))
            continue
        if n == "conv.time_enc.w.weight":
            # high-frequency encodings: fp32 w * dt has an ulp of ~0.25 rad at dt ~ 1e6, so cos/sin there
            # differ between any two implementations; compare the low-frequency dims
            ok = (pc.detach().abs().view(-1) * max_dt) < 1e3
            errs[n] = float((a.view(-1)[ok] - b.view(-1)[ok]).norm() / scale[ok].norm().float())
        else:
            errs[n] = float((a - b).norm() / (b.norm() + 1e-8))
    tol = {"conv.time_enc.w.weight": 2e-2, "conv.w_k.bias": 0.2}
    bad = {n: e for n, e in errs.items() if e > tol.get(n, TOL[precision]["grad"])}
    assert not bad, errs


def test_eval_and_predict_run(tmp_path):
    s = _session("cuda", tmp_path, runtime={"cuda_graphs": True})
    r = s.run_epoch("train")
    assert r["steps"] > 0 and r["loss"] > 0
    v = s.run_epoch("val")
    assert 0.0 <= v["metrics"]["ap"] <= 1.0
    p = s.predict("test")
    assert len(p.predictions) > 0


def _jodie_session(device, tmp_path, **over):
    from starry_unigraph import SchedulerSession

    cfg = _cfg(device, **over)
    cfg["model"].update({"name": "jodie", "family": "jodie"})
    s = SchedulerSession.from_config(cfg)
    s.ctx.artifact_root = tmp_path / ("jodie_" + device.replace(":", "_"))
    s.prepare_data()
    s.build_runtime()
    return s


@pytest.mark.parametrize("precision,edge_dtype", [("tf32", "fp32"), ("bf16", "fp32"), ("bf16", "bf16")])
def test_jodie_fused_step_matches_cpu_oracle(tmp_path, precision, edge_dtype):
    """JODIE (tanh-RNN memory + time projection): losses, predictions, memory and
    mailbox (lr = 0), then the gradients of the trainable parameters. With bf16
    edge features (the JODIE config's storage) the device keeps them in bf16 and
    the CPU path widens the same values."""
    tol = TOL[precision]
    data = {"synthetic": dict(_cfg("cpu")["data"]["synthetic"], edge_dtype=edge_dtype)}
    g = _jodie_session("cuda", tmp_path, train={"lr": 0.0}, runtime={"precision": precision}, data=data)
    c = _jodie_session("cpu", tmp_path, train={"lr": 0.0}, data=data)
    if edge_dtype == "bf16":
        assert g.ctdg_session.online_runtime.engine.efeat.dtype == torch.bfloat16
    rg, rc = g.ctdg_session.online_runtime, c.ctdg_session.online_runtime
    assert rg.engine is not None and rg.engine.kind == "jodie"
    eng = rg.engine
    for i, batch in enumerate(list(rc.iter_batches("train", 100))[:8]):
        res_g = rg.train_step(batch)
        neg = eng.neg[: batch.size].cpu()
        rc._negative_sample = lambda b, neg=neg: neg
        res_c = rc.train_step(batch)
        assert abs(res_g["loss"] - res_c["loss"]) <= tol["loss"] * max(1.0, abs(res_c["loss"])), \
            (i, res_g["loss"], res_c["loss"])
        pg, pc = torch.tensor(res_g["predictions"]), torch.tensor(res_c["predictions"])
        assert float((pg - pc).abs().max()) < tol["pred"], i
    from starry_unigraph.ops import check_status

    check_status()
    assert torch.allclose(rg.memory.memory.cpu(), rc.memory.memory, atol=tol["table"], rtol=tol["table"])
    assert torch.allclose(rg.memory.mailbox.cpu(), rc.memory.mailbox, atol=tol["table"], rtol=tol["table"])
    for (n, pg), pc in zip(rg.model.named_parameters(), rc.model.parameters()):
        a, b = pg.grad.detach().cpu(), pc.grad.detach()
        rel = float((a - b).norm() / (b.norm() + 1e-8))
        assert rel < tol["grad"], (n, rel)


def test_train_batches_matches_per_step_api(tmp_path):
    """The pipelined public API (async per-step H2D/D2H, one final sync) returns the
    same losses as stepping one batch at a time."""
    # lr = 0: gradient atomics (split-K flushes, concurrent weight-gradient streams) sum in a run-dependent
    # order, and Adam would turn those last-bit differences into diverging parameters
    a = _session("cuda", tmp_path / "a", runtime={"cuda_graphs": True}, train={"lr": 0.0})
    b = _session("cuda", tmp_path / "b", runtime={"cuda_graphs": True}, train={"lr": 0.0})
    batches = list(a.ctdg_session.online_runtime.iter_batches("train", 100))[:10]
    for x in batches:
        x.src, x.dst, x.ts, x.event_ids = (t.pin_memory() for t in (x.src, x.dst, x.ts, x.event_ids))
    la = [a.ctdg_session.train_step(x)["loss"] for x in batches]
    lb = [r["loss"] for r in b.ctdg_session.train_batches(batches)]
    torch.testing.assert_close(torch.tensor(lb), torch.tensor(la), rtol=1e-4, atol=1e-5)
