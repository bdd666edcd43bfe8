"""Worker for the two-rank CommEngine test (gloo): owner-routed exchange, remote
fetch, delta push / poll and the gradient all-reduce (exact and int8), checked
against values every rank can compute locally; writes outcome_r<rank>.json.

    python -m torch.distributed.run --nproc-per-node 2 ... comm_engine_worker.py --out DIR
"""
import argparse
import datetime
import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--out", required=True)
    a = p.parse_args()
    import torch
    import torch.distributed as dist

    from starry_unigraph.runtime.comm.comm_engine import CommEngine

    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    rank, W = dist.get_rank(), dist.get_world_size()
    N, F = 20, 3
    owner = torch.arange(N) % W
    full = torch.arange(N * F, dtype=torch.float32).view(N, F)  # row v = the owner's row of node v
    table = torch.where((owner == rank).unsqueeze(1), full, torch.full_like(full, -1.0))  # only owned rows valid
    ce = CommEngine(owner=owner, rank=rank)
    checks = {}
    # exchange: every rank sends rows of ids 3r..3r+5; each owner receives exactly its ids
    ids = torch.arange(3 * rank, 3 * rank + 6)
    r_ids, r_rows = ce.async_exchange(ids, full[ids] + 1000 * rank).wait()
    sent = {(r, v) for r in range(W) for v in range(3 * r, 3 * r + 6) if v % W == rank}
    got = {(int(round(float(row[0] - full[v, 0]) / 1000)), int(v)) for v, row in zip(r_ids.tolist(), r_rows)}
    checks["exchange"] = got == sent
    # fetch: rows of arbitrary (also remote, repeated) ids come back from their owners
    want = torch.tensor([7, 0, 13, 7, 2 + rank, 19])
    checks["fetch"] = bool(torch.equal(ce.async_fetch(want, table).wait(), full[want]))
    # delta push / poll
    ce.push_delta(torch.tensor([rank, rank + 2]), torch.ones(2, F) * (rank + 1))
    d = ce.try_recv_delta()
    checks["delta"] = d is not None and bool((owner[d[0]] == rank).all()) and ce.try_recv_delta() is None
    # gradient all-reduce: exact mean, and int8 within one quantisation step
    g = torch.Generator().manual_seed(rank)
    w = torch.nn.Parameter(torch.zeros(4, 5))
    w.grad = torch.randn(4, 5, generator=g)
    grads = [torch.randn(4, 5, generator=torch.Generator().manual_seed(r)) for r in range(W)]
    ce.all_reduce_gradients([w])
    checks["allreduce"] = bool(torch.allclose(w.grad, sum(grads) / W, atol=1e-6))
    w.grad = grads[rank].clone()
    CommEngine(owner=owner, rank=rank, int8_gradients=True).all_reduce_gradients([w])
    step = max(float(x.abs().max()) for x in grads) / 127.0
    checks["int8"] = bool(((w.grad - sum(grads) / W).abs() <= step).all())
    (Path(a.out) / f"outcome_r{rank}.json").write_text(json.dumps(checks))
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
