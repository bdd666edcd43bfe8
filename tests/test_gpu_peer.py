"""NVLink peer kernels on one GPU, with the ranks' buffers emulated as separate
local allocations (no kernel waits on another kernel): barrier signalling and
its bounded timeout, the fused all-reduce + Adam, CTDG memory write-back and
the mailbox claim/write protocol."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from starry_unigraph.ops import cuda_ext

    return cuda_ext()


def _table(*ts):
    return torch.tensor([t.data_ptr() for t in ts], dtype=torch.int64, device="cuda")


def test_barrier_signals_peers_and_times_out_boundedly():
    from starry_unigraph.ops import check_status

    C = _C()
    f0 = torch.zeros(32, dtype=torch.int64, device="cuda")  # rank 0's flag array
    f1 = torch.zeros(32, dtype=torch.int64, device="cuda")  # "rank 1"'s flag array
    f0[1] = 1  # rank 1 already reached barrier epoch 1
    epoch = torch.zeros(1, dtype=torch.int64, device="cuda")
    C.peer_barrier(_table(f0, f1), 0, 2, epoch, 50_000_000)
    torch.cuda.synchronize()
    check_status()
    assert int(f1[0]) == 1 and int(epoch) == 1
    # epoch 2: nothing ever sets f0[1] = 2 -> the wait gives up and reports
    C.peer_barrier(_table(f0, f1), 0, 2, epoch, 2_000_000)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="peer flag"):
        check_status()
    assert int(f1[0]) == 2


def test_allreduce_adam_matches_torch():
    C = _C()
    n = 4096 + 4
    torch.manual_seed(0)
    g = [torch.randn(n, device="cuda") for _ in range(3)]
    p = torch.randn(n, device="cuda")
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    step = torch.zeros(1, dtype=torch.int64, device="cuda")
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    ref = p.clone().requires_grad_(True)
    opt = torch.optim.Adam([ref], lr=1e-2)
    for it in range(3):
        C.peer_allreduce_adam(_table(*g), 3, p, m, v, step, done, 1e-2, 0.9, 0.999, 1e-8, 0.0, 1.0 / 3)
        ref.grad = (g[0] + g[1] + g[2]) / 3
        opt.step()
        for x in g:
            x.mul_(0.5)
    torch.cuda.synchronize()
    assert int(step) == 3
    torch.testing.assert_close(p, ref.detach(), rtol=1e-5, atol=1e-6)


def test_memory_writeback_and_mail_claims():
    C = _C()
    N, D, E = 10, 8, 4
    SW = 2 * D + E
    owner = (torch.arange(N, device="cuda") % 2).int()
    mem = [torch.zeros(N, D, device="cuda") for _ in range(2)]
    mts = [torch.full((N,), -1.0, device="cuda") for _ in range(2)]
    mail = [torch.zeros(N, SW, device="cuda") for _ in range(2)]
    mail_ts = [torch.zeros(N, device="cuda") for _ in range(2)]
    claim = [torch.zeros(N, dtype=torch.int64, device="cuda") for _ in range(2)]
    efeat = torch.randn(50, E, device="cuda")

    def rank_step(roots, ts_max, ev, fill):
        R = len(roots)
        r = torch.tensor(roots, dtype=torch.int64, device="cuda")
        nr = torch.tensor([R], dtype=torch.int32, device="cuda")
        mem_new = torch.full((R, D), fill, device="cuda")
        C.tgn_peer_writeback(r, nr, mem_new, owner, _table(*mem), _table(*mts),
                             torch.tensor([ts_max], device="cuda"))
        # one event per root: root i is the source of event i, its destination is root (i + 1) % R
        win = torch.cat([torch.arange(R), torch.full((R,), -1)]).int().cuda()
        src_idx = torch.arange(R, dtype=torch.int32, device="cuda")
        dst_idx = ((torch.arange(R) + 1) % R).int().cuda()
        eid = torch.tensor([e for e, _ in ev], dtype=torch.int64, device="cuda")
        ets = torch.tensor([t for _, t in ev], dtype=torch.float32, device="cuda")
        mem_prev = torch.full((R, D), fill, device="cuda")
        return dict(r=r, nr=nr, win=win, src_idx=src_idx, dst_idx=dst_idx, eid=eid, ets=ets, mem_prev=mem_prev)

    a = rank_step([0, 1, 2], 5.0, [(10, 4.0), (11, 5.0), (12, 5.0)], 1.0)
    b = rank_step([1, 3], 7.0, [(20, 3.0), (21, 7.0)], 2.0)
    for x in (a, b):
        C.tgn_peer_mail_claim(x["r"], x["nr"], x["win"], x["eid"], x["ets"], owner, _table(*claim))
    for x in (a, b):
        C.tgn_peer_mail_write(x["r"], x["nr"], x["win"], x["src_idx"], x["dst_idx"], x["eid"], x["ets"],
                              x["mem_prev"], efeat, E, owner, _table(*claim), _table(*mail), _table(*mail_ts))
    torch.cuda.synchronize()
    # memory rows land on the owner; memory_ts is the max over writers
    assert torch.equal(mem[0][0], torch.ones(D, device="cuda")) and torch.equal(mem[0][2], torch.ones(D, device="cuda"))
    assert float(mts[1][1]) == 7.0 and float(mts[1][3]) == 7.0 and float(mts[0][0]) == 5.0
    assert float(mem[1][3][0]) == 2.0
    # node 1: rank a proposes (ts 5, eid 11), rank b (ts 3, eid 20) -> a's mail wins
    assert float(mail_ts[1][1]) == 5.0 and float(mail[1][1][0]) == 1.0
    assert torch.equal(mail[1][1][2 * D:], efeat[11])
    assert float(mail_ts[1][3]) == 7.0 and torch.equal(mail[1][3][2 * D:], efeat[21])
    assert float(mail_ts[0][2]) == 5.0 and torch.equal(mail[0][2][2 * D:], efeat[12])


def test_writeback_historical_filter():
    """Rank 0 pushes rows of nodes owned by rank 1 through the historical cache:
    a first push always lands, a row within the cosine threshold of the cached one
    is dropped, a row beyond it lands and refreshes the cache; rank 0's own nodes
    are never filtered."""
    C = _C()
    N, D = 6, 16
    owner = (torch.arange(N, device="cuda") % 2).int()
    mem = [torch.zeros(N, D, device="cuda") for _ in range(2)]
    mts = [torch.full((N,), -1.0, device="cuda") for _ in range(2)]
    shared = owner != 0
    slot_of = torch.full((N,), -1, dtype=torch.int64, device="cuda")
    slot_of[shared] = torch.arange(int(shared.sum()), device="cuda")
    cache = [slot_of, torch.zeros(int(shared.sum()), D, device="cuda"),
             torch.full((int(shared.sum()),), -1.0, device="cuda")]
    base = torch.randn(D, device="cuda")

    def push(rows, ts):
        r = torch.tensor([1, 0], dtype=torch.int64, device="cuda")  # node 1 (rank 1's), node 0 (own)
        C.tgn_peer_writeback(r, torch.tensor([2], dtype=torch.int32, device="cuda"), torch.stack(rows), owner,
                             _table(*mem), _table(*mts), torch.tensor([ts], device="cuda"), cache, 0.5, 0)
        torch.cuda.synchronize()

    push([base, base], 1.0)                                   # never pushed: lands
    assert torch.equal(mem[1][1], base) and float(mts[1][1]) == 1.0
    near = base + 0.01 * torch.randn(D, device="cuda")        # cos distance ~ 1e-4 < 0.5: dropped
    push([near, near], 2.0)
    assert torch.equal(mem[1][1], base) and float(mts[1][1]) == 1.0
    assert torch.equal(mem[0][0], near) and float(mts[0][0]) == 2.0  # own node: always written
    far = -base                                               # cos distance 2 > 0.5: lands, cache refreshed
    push([far, far], 3.0)
    assert torch.equal(mem[1][1], far) and float(mts[1][1]) == 3.0
    assert torch.equal(cache[1][int(slot_of[1])], far) and float(cache[2][int(slot_of[1])]) == 3.0


def test_sharded_memory_reads_match_local_table():
    """The attention projections with node memory split over two emulated owner
    tables (peer descriptor) equal the same projections on the full table, with
    this step's roots read from the fresh-row buffer when stamped."""
    C = _C()
    torch.manual_seed(0)
    N, D, E, T, Do, k, R = 64, 32, 8, 16, 32, 5, 24
    dev = "cuda"
    mem_full = torch.randn(N, D, device=dev)
    owner = (torch.arange(N, device=dev) % 2).int()
    tables = [torch.zeros(N, D, device=dev) for _ in range(2)]
    for q in range(2):
        tables[q][owner == q] = mem_full[owner == q]
    roots = torch.randperm(N, device=dev)[:R].long()
    n_roots = torch.tensor([R], dtype=torch.int32, device=dev)
    nbr = torch.randint(0, N, (R * k,), device=dev)
    nbr_eid = torch.randint(0, 50, (R * k,), device=dev)
    nbr_dt = torch.rand(R * k, device=dev) * 1e4
    nbr_cnt = torch.full((R,), k, dtype=torch.int32, device=dev)
    efeat = torch.randn(50, E, device=dev)
    te_w, te_b = torch.randn(T, device=dev), torch.randn(T, device=dev)
    wq, bq = torch.randn(Do, D + T, device=dev), torch.randn(Do, device=dev)
    wk, bk = torch.randn(Do, D + E + T, device=dev), torch.randn(Do, device=dev)
    wv, bv = torch.randn(Do, D + E + T, device=dev), torch.randn(Do, device=dev)
    Q0, KV0 = torch.zeros(R, Do, device=dev), torch.zeros(R * k, 2 * Do, device=dev)
    C.tgn_attn_proj(mem_full, roots, n_roots, nbr, nbr_eid, nbr_dt, nbr_cnt, efeat, E, te_w, te_b, wq, bq, wk, bk,
                    wv, bv, Q0, KV0, None)
    # peer view: rows from the owners' tables; stamps never match the step tag -> no fresh rows
    stamp = torch.zeros(N, dtype=torch.int32, device=dev)
    node2root = torch.zeros(N, dtype=torch.int32, device=dev)
    step = torch.full((1,), 7, dtype=torch.int64, device=dev)
    mem_new = torch.zeros(R, D, device=dev)
    desc = torch.tensor([_table(*tables).data_ptr(), 0, owner.data_ptr(), stamp.data_ptr(), node2root.data_ptr(),
                         step.data_ptr(), mem_new.data_ptr(), 0], dtype=torch.int64)
    keep = _table(*tables)  # keep the pointer table alive
    desc[0] = keep.data_ptr()
    Q1, KV1 = torch.zeros_like(Q0), torch.zeros_like(KV0)
    C.tgn_attn_proj(torch.zeros(N, D, device=dev), roots, n_roots, nbr, nbr_eid, nbr_dt, nbr_cnt, efeat, E, te_w,
                    te_b, wq, bq, wk, bk, wv, bv, Q1, KV1, desc)
    torch.cuda.synchronize()
    torch.testing.assert_close(Q1, Q0)
    torch.testing.assert_close(KV1, KV0)
    # stamped roots come from mem_new (tag = ((step - 1) & 0x3FFFFFFF) + 1 = 7)
    stamp[roots] = 7
    node2root[roots] = torch.arange(R, dtype=torch.int32, device=dev)
    mem_new.copy_(mem_full[roots] * 2.0)
    C.tgn_attn_proj(torch.zeros(N, D, device=dev), roots, n_roots, nbr, nbr_eid, nbr_dt, nbr_cnt, efeat, E, te_w,
                    te_b, wq, bq, wk, bk, wv, bv, Q1, KV1, desc)
    mem_ref = mem_full.clone()
    mem_ref[roots] = mem_full[roots] * 2.0
    C.tgn_attn_proj(mem_ref, roots, n_roots, nbr, nbr_eid, nbr_dt, nbr_cnt, efeat, E, te_w, te_b, wq, bq, wk, bk,
                    wv, bv, Q0, KV0, None)
    torch.cuda.synchronize()
    torch.testing.assert_close(Q1, Q0)
    torch.testing.assert_close(KV1, KV0)


def test_halo_gather_and_push_kernels():
    """Aggregation reading source rows from two emulated ranks' staging buffers,
    and its transposed push, against dense references."""
    C = _C()
    torch.manual_seed(1)
    F, n_dst, n_src = 64, 40, 70
    src_owner = torch.randint(0, 2, (n_src,), dtype=torch.int32, device="cuda")
    src_row = torch.zeros(n_src, dtype=torch.int32, device="cuda")
    counts = [0, 0]
    for i, o in enumerate(src_owner.tolist()):
        src_row[i] = counts[o]
        counts[o] += 1
    stages = [torch.zeros(max(counts), F, device="cuda") for _ in range(2)]
    x_src = torch.randn(n_src, F, device="cuda")
    for i, (o, r) in enumerate(zip(src_owner.tolist(), src_row.tolist())):
        stages[o][r] = x_src[i]
    E = 400
    src = torch.randint(0, n_src, (E,), device="cuda")
    dst = torch.randint(0, n_dst, (E,), device="cuda")
    val = torch.rand(E, device="cuda")
    order = torch.argsort(dst, stable=True)
    rowptr = torch.zeros(n_dst + 1, dtype=torch.int64, device="cuda")
    rowptr[1:] = torch.cumsum(torch.bincount(dst, minlength=n_dst), 0)
    out = C.spmm_peer_gather(rowptr, src[order].int().contiguous(), val[order].contiguous(), _table(*stages),
                             src_owner, src_row, n_dst, F)
    ref = torch.zeros(n_dst, F, device="cuda").index_add_(0, dst, x_src[src] * val[:, None])
    torch.testing.assert_close(out, ref, rtol=1e-5, atol=1e-5)
    # pull-once form: rank 0's view, the rows owned by rank 1 are pulled into a
    # local halo table and the aggregation reads [rank 0's rows | halo rows]
    remote = src_owner != 0
    halo_src = torch.nonzero(remote).view(-1).int()
    halo = C.halo_pull(_table(*stages), src_owner, src_row, halo_src, F)
    torch.testing.assert_close(halo, x_src[halo_src.long()])
    slot = torch.cumsum(remote.int(), 0) - 1
    remap = torch.where(remote, counts[0] + slot, src_row.long())
    col2 = remap[src[order]].int().contiguous()
    out2 = C.spmm_two_tables(rowptr, col2, val[order].contiguous(), stages[0][: counts[0]].contiguous(), halo, n_dst)
    torch.testing.assert_close(out2, ref, rtol=1e-5, atol=1e-5)
    # local rows read in place from a wider staging buffer (row stride 2F + 4)
    wide = torch.zeros(counts[0], 2 * F + 4, device="cuda")
    wide[:, :F] = stages[0][: counts[0]]
    out3 = C.spmm_two_tables(rowptr, col2, val[order].contiguous(), wide[:, :F], halo, n_dst)
    torch.testing.assert_close(out3, ref, rtol=1e-5, atol=1e-5)
    # backward push: grad of source rows lands in the owners' buffers
    g = torch.randn(n_dst, F, device="cuda")
    order_t = torch.argsort(src, stable=True)
    rowptr_t = torch.zeros(n_src + 1, dtype=torch.int64, device="cuda")
    rowptr_t[1:] = torch.cumsum(torch.bincount(src, minlength=n_src), 0)
    gbufs = [torch.zeros_like(s) for s in stages]
    C.spmm_peer_push(rowptr_t, dst[order_t].int().contiguous(), val[order_t].contiguous(), g, n_src,
                     _table(*gbufs), src_owner, src_row)
    gref = torch.zeros(n_src, F, device="cuda").index_add_(0, src, g[dst] * val[:, None])
    got = torch.stack([gbufs[o][r] for o, r in zip(src_owner.tolist(), src_row.tolist())])
    torch.testing.assert_close(got, gref, rtol=1e-5, atol=1e-5)


def test_rs_adam_ag_matches_torch_on_every_replica():
    """Reduce-scatter + Adam + all-gather, three ranks emulated by three launches:
    every replica ends with the torch Adam result of the mean gradient, each rank
    having updated only its own shard."""
    C = _C()
    W, n = 3, 4096 + 12
    torch.manual_seed(0)
    g = [torch.randn(n, device="cuda") for _ in range(W)]
    p0 = torch.randn(n, device="cuda")
    params = [p0.clone() for _ in range(W)]
    mv = [(torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")) for _ in range(W)]
    steps = [torch.zeros(1, dtype=torch.int64, device="cuda") for _ in range(W)]
    dones = [torch.zeros(1, dtype=torch.int32, device="cuda") for _ in range(W)]
    gt, pt = _table(*g), _table(*params)
    ref = p0.clone().requires_grad_(True)
    opt = torch.optim.Adam([ref], lr=1e-2)
    for it in range(3):
        for r in range(W):
            C.peer_rs_adam_ag(gt, pt, W, r, params[r], mv[r][0], mv[r][1], steps[r], dones[r], 1e-2, 0.9, 0.999,
                              1e-8, 0.0, 1.0 / W)
        ref.grad = sum(g) / W
        opt.step()
        for x in g:
            x.mul_(0.5)
    torch.cuda.synchronize()
    assert all(int(s) == 3 for s in steps)
    for r in range(W):
        torch.testing.assert_close(params[r], ref.detach(), rtol=1e-5, atol=1e-6)
    assert torch.equal(params[0], params[1]) and torch.equal(params[1], params[2])


def test_wait_claim_and_push():
    """The end-of-step protocol on two emulated ranks: the fused wait + claim
    (peers' flags already at the epoch, so the wait passes), then one push per
    rank (memory write-back + the claim winners' mailbox slots); the end-of-step
    signal stores the next epoch into the peer's flag array."""
    C = _C()
    N, D, E = 10, 8, 4
    SW = 2 * D + E
    owner = (torch.arange(N, device="cuda") % 2).int()
    mem = [torch.zeros(N, D, device="cuda") for _ in range(2)]
    mts = [torch.full((N,), -1.0, device="cuda") for _ in range(2)]
    mail = [torch.zeros(N, SW, device="cuda") for _ in range(2)]
    mail_ts = [torch.zeros(N, device="cuda") for _ in range(2)]
    claim = [torch.zeros(N, dtype=torch.int64, device="cuda") for _ in range(2)]
    flags = [torch.zeros(32, dtype=torch.int64, device="cuda") for _ in range(2)]
    epochs = [torch.ones(1, dtype=torch.int64, device="cuda") for _ in range(2)]
    flags[0][1] = 1
    flags[1][0] = 1
    efeat = torch.randn(50, E, device="cuda")

    def rank_data(roots, ts_max, ev, fill):
        R = len(roots)
        return dict(r=torch.tensor(roots, dtype=torch.int64, device="cuda"),
                    nr=torch.tensor([R], dtype=torch.int32, device="cuda"),
                    mem_new=torch.full((R, D), fill, device="cuda"), ts_max=torch.tensor([ts_max], device="cuda"),
                    win=torch.cat([torch.arange(R), torch.full((R,), -1)]).int().cuda(),
                    src_idx=torch.arange(R, dtype=torch.int32, device="cuda"),
                    dst_idx=((torch.arange(R) + 1) % R).int().cuda(),
                    eid=torch.tensor([e for e, _ in ev], dtype=torch.int64, device="cuda"),
                    ets=torch.tensor([t for _, t in ev], dtype=torch.float32, device="cuda"),
                    mem_prev=torch.full((R, D), fill, device="cuda"))

    data = [rank_data([0, 1, 2], 5.0, [(10, 4.0), (11, 5.0), (12, 5.0)], 1.0),
            rank_data([1, 3], 7.0, [(20, 3.0), (21, 7.0)], 2.0)]
    for q, x in enumerate(data):
        C.tgn_peer_wait_claim(flags[q], q, 2, epochs[q], 50_000_000, x["r"], x["nr"], x["win"], x["eid"], x["ets"],
                              owner, _table(*claim))
    for q, x in enumerate(data):
        C.tgn_peer_push(x["r"], x["nr"], x["mem_new"], x["ts_max"], owner, _table(*mem), _table(*mts), None, 0.5, q,
                        x["win"], x["src_idx"], x["dst_idx"], x["eid"], x["ets"], x["mem_prev"], efeat, E,
                        _table(*claim), _table(*mail), _table(*mail_ts))
    C.peer_signal(_table(*flags), 0, 2, epochs[0])
    torch.cuda.synchronize()
    from starry_unigraph.ops import check_status

    check_status()
    assert int(flags[1][0]) == 2 and int(epochs[0]) == 2
    assert torch.equal(mem[0][0], torch.ones(D, device="cuda")) and torch.equal(mem[0][2], torch.ones(D, device="cuda"))
    assert float(mts[1][1]) == 7.0 and float(mts[1][3]) == 7.0 and float(mts[0][0]) == 5.0
    assert float(mem[1][3][0]) == 2.0
    # node 1: rank 0 proposes (ts 5, eid 11), rank 1 (ts 3, eid 20) -> rank 0's mail wins
    assert float(mail_ts[1][1]) == 5.0 and float(mail[1][1][0]) == 1.0
    assert torch.equal(mail[1][1][2 * D:], efeat[11])
    assert float(mail_ts[1][3]) == 7.0 and torch.equal(mail[1][3][2 * D:], efeat[21])
    assert float(mail_ts[0][2]) == 5.0 and torch.equal(mail[0][2][2 * D:], efeat[12])
    # bf16 edge features give the same slot values as their fp32 copies
    mail_b = [torch.zeros_like(m) for m in mail]
    mts_b = [torch.zeros_like(m) for m in mail_ts]
    mem_b = [torch.zeros_like(m) for m in mem]
    ets_b = [torch.full_like(m, -1.0) for m in mts]
    ef_b = efeat.bfloat16()
    for q, x in enumerate(data):
        C.tgn_peer_push(x["r"], x["nr"], x["mem_new"], x["ts_max"], owner, _table(*mem_b), _table(*ets_b), None, 0.5,
                        q, x["win"], x["src_idx"], x["dst_idx"], x["eid"], x["ets"], x["mem_prev"], ef_b, E,
                        _table(*claim), _table(*mail_b), _table(*mts_b))
    torch.cuda.synchronize()
    assert torch.equal(mail_b[1][3][2 * D:], ef_b[21].float())
