"""Fused compute + NVLink paths timed in isolation, each against its NCCL form.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N --master-addr 127.0.0.1 \\
        --master-port P bench_fused.py [--iters 50] [--warmup 5]

Rank 0 prints one JSON line per path and size:

* ``allreduce_adam``: the data-parallel gradient all-reduce fused with Adam
  (``PeerAllReduceAdam``: device barrier, one kernel in which rank r sums shard r
  of all W gradient buffers in rank order over NVLink, applies Adam to it and
  stores the new shard into every rank's parameters, barrier) against
  ``dist.all_reduce`` (NCCL) followed by the fused Adam kernel.
  ``all_read_us`` times the earlier form in which every rank reads all W
  gradient buffers whole and updates all parameters itself.
* ``halo_gather``: the DTDG halo exchange of ``halo_aggregate`` (staging copy,
  device barrier, each halo row pulled once from its owner over NVLink, SpMM
  over [own | halo] rows) against the reference's scheme: gather the boundary
  rows each peer asked for, ``dist.all_to_all_single`` (NCCL), then the local
  SpMM over [own | halo] rows. ``per_edge_pull_us`` times the other peer form,
  where the SpMM reads every halo edge's source row from the owner.
* ``writeback`` (TGN shape): the CTDG memory write-back + mail write of one step
  (``tgn_peer_push``) against rows grouped by owner, ``all_to_all_single`` and a
  local index copy.
* ``remote_fetch`` (TGN shape): the attention projections reading node memory
  from the owners' tables inside the operand producer (``tgn_attn_proj`` with a
  peer descriptor) against fetching the remote rows with ``all_to_all_single``
  into a local replica first.

Times are device times (CUDA events on the launching stream, synchronised on
both sides), max over ranks. ``nvlink_bytes`` is what one rank must pull over
NVLink; the roofline time is the slower of those bytes at the measured
peer-copy bandwidth (770 GB/s per direction on this pool's NVLink 5) and the
rank's local HBM bytes at the measured copy bandwidth (``hbm_gbs`` of
MEASURED_PEAKS.json next to this file, else 6550 GB/s); ``frac`` is the
roofline time over the measured time.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import torch
import torch.distributed as dist

NVLINK_GBS = 770.0


def _hbm_gbs() -> float:
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6550.0


def _time(fn, iters: int, warmup: int) -> float:
    """Mean device ms per call, max over ranks."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    t = torch.tensor([s.elapsed_time(e) / iters], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _report(path: str, size: dict, fused_ms: float, nccl_ms: float, nvlink_bytes: float, hbm_bytes: float,
            world: int) -> dict:
    roof_ms = max(nvlink_bytes / (NVLINK_GBS * 1e9), hbm_bytes / (_hbm_gbs() * 1e9)) * 1e3
    return {"path": path, "n_gpus": world, **size, "fused_us": round(fused_ms * 1e3, 2),
            "nccl_us": round(nccl_ms * 1e3, 2), "speedup_vs_nccl": round(nccl_ms / fused_ms, 3),
            "nvlink_bytes_per_rank": int(nvlink_bytes),
            "nvlink_gbs": round(nvlink_bytes / (fused_ms * 1e-3) / 1e9, 1),
            "roofline_us": round(roof_ms * 1e3, 2), "frac": round(roof_ms / fused_ms, 3)}


def bench_allreduce_adam(n: int, iters: int, warmup: int, C) -> dict:
    from starry_unigraph.parallel.ctdg_peer import DEFAULT_BARRIER_BUDGET
    from starry_unigraph.parallel.symmetric import SymmetricArena

    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    n = (n + 3) // 4 * 4
    arena = SymmetricArena({"grad": ((n,), torch.float32), "param": ((n,), torch.float32),
                            "flags": ((32,), torch.int64)}, dev)
    g = arena["grad"]
    g.normal_(generator=torch.Generator(device=dev).manual_seed(rank))
    arena["flags"].zero_()
    p = arena["param"]
    p.normal_(generator=torch.Generator(device=dev).manual_seed(99))  # same on every rank
    tg, tp, tf = arena.peer_table("grad"), arena.peer_table("param"), arena.peer_table("flags")
    m, v = torch.zeros_like(p), torch.zeros_like(p)
    step = torch.zeros(1, dtype=torch.int64, device=dev)
    done = torch.zeros(1, dtype=torch.int32, device=dev)
    epoch = torch.zeros(1, dtype=torch.int64, device=dev)
    torch.cuda.synchronize()
    arena.barrier_host()

    def fused():
        C.peer_barrier(tf, rank, world, epoch, DEFAULT_BARRIER_BUDGET)
        C.peer_rs_adam_ag(tg, tp, world, rank, p, m, v, step, done, 1e-6, 0.9, 0.999, 1e-8, 0.0, 1.0 / world)
        C.peer_barrier(tf, rank, world, epoch, DEFAULT_BARRIER_BUDGET)

    p2 = torch.randn(n, device=dev)

    def all_read():
        C.peer_barrier(tf, rank, world, epoch, DEFAULT_BARRIER_BUDGET)
        C.peer_allreduce_adam(tg, world, p2, m, v, step, done, 1e-6, 0.9, 0.999, 1e-8, 0.0, 1.0 / world)
        C.peer_barrier(tf, rank, world, epoch, DEFAULT_BARRIER_BUDGET)

    g2 = torch.randn(n, device=dev)

    def nccl():
        dist.all_reduce(g2)
        C.adam_flat(p2, g2, m, v, step, done, 1e-6, 0.9, 0.999, 1e-8, 0.0, 1.0 / world)

    fused_ms = _time(fused, iters, warmup)
    all_read_ms = _time(all_read, iters, warmup)
    nccl_ms = _time(nccl, iters, warmup)
    # replicas must hold the same parameters after the fused steps
    ref = p.clone()
    dist.broadcast(ref, src=0)
    same = bool(torch.equal(ref, p))
    # per rank: pull shard r of the W-1 remote gradient buffers, push the new shard into
    # the W-1 remote parameter buffers (each direction (W-1)/W * n * 4 bytes); locally
    # read its own gradient shard, p, m, v and write p, m, v of the shard
    nvl = (world - 1) * (n // world) * 4.0
    hbm = 7 * (n // world) * 4.0
    r = _report("allreduce_adam", {"numel": n}, fused_ms, nccl_ms, nvl, hbm, world)
    r["all_read_us"] = round(all_read_ms * 1e3, 2)
    r["replicas_equal"] = same
    return r


def bench_halo_gather(n: int, m: int, F: int, iters: int, warmup: int, C) -> dict:
    from starry_unigraph.data.partition import NID, SnapshotBlock
    from starry_unigraph.parallel.halo import PeerHaloContext, halo_aggregate, set_halo_context

    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    # contiguous node blocks per rank; this rank's destination rows get m / W edges
    # with uniformly random sources, so (W-1)/W of them come from halo rows. The
    # block's source rows are [this rank's nodes | its unique halo nodes], the
    # layout of the partitioned snapshot blocks.
    parts = torch.arange(n) * world // n
    lo = int((parts < rank).sum())
    n_local = int((parts == rank).sum())
    gen = torch.Generator().manual_seed(1234 + rank)
    me = m // world
    dst = torch.randint(0, n_local, (me,), generator=gen)
    src = torch.randint(0, n, (me,), generator=gen)
    val = torch.rand(me, generator=gen)
    is_remote = parts[src] != rank
    halo = torch.unique(src[is_remote])  # sorted, hence grouped by owner
    src_nodes = torch.cat([torch.arange(lo, lo + n_local), halo])
    pos = torch.full((n,), -1, dtype=torch.long)
    pos[src_nodes] = torch.arange(src_nodes.numel())
    block = SnapshotBlock(num_src_nodes=int(src_nodes.numel()), num_dst_nodes=n_local,
                          edge_src=pos[src].to(dev), edge_dst=dst.to(dev), srcdata={NID: src_nodes.to(dev)},
                          edata={"gcn_norm": val.to(dev)})
    csr = block.csr()
    x_local = torch.randn(n_local, F, device=dev)
    hc = PeerHaloContext(parts, F, dev)
    set_halo_context(hc)
    owner, row = hc.src_maps(block)

    def fused():
        with torch.no_grad():
            return halo_aggregate(block, x_local)

    calls = [0]

    def per_edge():  # every halo edge reads its source row from the owner
        k = calls[0] % 2
        calls[0] += 1
        hc.arena[f"x{k}"][:n_local].copy_(x_local)
        hc.barrier()
        return C.spmm_peer_gather(csr["rowptr"], csr["col"], csr["val"], hc.tables[f"x{k}"], owner, row,
                                  n_local, F)

    # NCCL form (reference Route.forward): halo rows requested once (setup), then
    # every call gathers the rows the peers asked for, exchanges them with one
    # all_to_all and aggregates over [own rows | received halo rows]
    recv_counts = torch.bincount(parts[halo], minlength=world)
    sc = torch.empty(world, dtype=torch.long, device=dev)
    dist.all_to_all_single(sc, recv_counts.to(dev))
    send_counts = sc.cpu()
    asked = torch.empty(int(send_counts.sum()), dtype=torch.long, device=dev)
    dist.all_to_all_single(asked, halo.to(dev), output_split_sizes=send_counts.tolist(),
                           input_split_sizes=recv_counts.tolist())
    send_idx = asked - lo
    ext = torch.empty(n_local + halo.numel(), F, device=dev)
    recv = torch.empty(halo.numel(), F, device=dev)
    sizes_s, sizes_r = send_counts.tolist(), recv_counts.tolist()

    def nccl():
        sendbuf = x_local.index_select(0, send_idx)
        dist.all_to_all_single(recv, sendbuf, output_split_sizes=sizes_r, input_split_sizes=sizes_s)
        ext[:n_local].copy_(x_local)
        ext[n_local:].copy_(recv)
        return C.spmm_csr(csr["rowptr"], csr["col"], csr["val"], ext, n_local, None, False, csr.get("plan"))

    a, b, c = fused(), nccl(), per_edge()
    torch.cuda.synchronize()
    err = max(float((a - b).abs().max()), float((c - b).abs().max()))
    fused_ms = _time(fused, iters, warmup)
    nccl_ms = _time(nccl, iters, warmup)
    per_edge_ms = _time(per_edge, iters, warmup)
    set_halo_context(None)
    remote_edges = int(is_remote.sum())
    nvl = halo.numel() * F * 4.0  # each halo row crosses NVLink once
    # staging copy (read + write), layer input rows read by the aggregation, halo
    # rows written and read back, CSR (8 B per edge), output
    hbm = (2 * n_local * F + n_local * F + 2 * halo.numel() * F + n_local * F) * 4.0 + me * 8.0
    r = _report("halo_gather", {"nodes": n, "edges": m, "F": F, "remote_edges_per_rank": remote_edges,
                                "unique_halo_rows_per_rank": int(halo.numel())},
                fused_ms, nccl_ms, nvl, hbm, world)
    r["per_edge_pull_us"] = round(per_edge_ms * 1e3, 2)
    r["max_abs_diff_vs_nccl"] = err
    return r


def _ctdg_batch(N: int, events: int, D: int, rank: int, dev):
    """One rank's synthetic CTDG step: `events` events with random endpoints, the
    roots (sources, destinations, one negative per event), each root's latest
    event as source / destination (`win`), and the rows the kernels read."""
    g = torch.Generator().manual_seed(4321 + rank)
    src = torch.randint(0, N, (events,), generator=g)
    dst = torch.randint(0, N, (events,), generator=g)
    neg = torch.randint(0, N, (events,), generator=g)
    roots, inv = torch.unique(torch.cat([src, dst, neg]), return_inverse=True)
    R = roots.numel()
    src_idx, dst_idx = inv[:events], inv[events:2 * events]
    ev = torch.arange(events)
    win = torch.full((2 * R,), -1, dtype=torch.long)
    win[:R].scatter_reduce_(0, src_idx, ev, "amax")
    win[R:].scatter_reduce_(0, dst_idx, ev, "amax")
    ev_ts = torch.sort(torch.rand(events, generator=g) * 1e6).values
    return dict(roots=roots.to(dev), n_roots=torch.tensor([R], dtype=torch.int32, device=dev), R=R,
                src_idx=src_idx.int().to(dev), dst_idx=dst_idx.int().to(dev), win=win.int().to(dev),
                ev_eid=(ev + rank * events).to(dev), ev_ts=ev_ts.to(dev),
                mem_new=torch.randn(R, D, device=dev), mem_prev=torch.randn(R, D, device=dev),
                ts_max=torch.tensor([float(ev_ts.max())], device=dev))


def bench_writeback(N: int, events: int, D: int, E: int, iters: int, warmup: int, C) -> dict:
    """Fused path #2: the memory write-back and mail write of one CTDG step
    (``tgn_peer_push``: each root's new memory row stored into its owner's table
    over NVLink, the claim winners' mailbox slots written in the same kernel),
    against the NCCL form: rows grouped by owner, ``all_to_all_single``, then a
    local index copy into the tables."""
    from starry_unigraph.parallel.symmetric import SymmetricArena

    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    SW = 2 * D + E
    arena = SymmetricArena({"memory": ((N, D), torch.float32), "memory_ts": ((N,), torch.float32),
                            "mailbox": ((N, SW), torch.float32), "mailbox_ts": ((N,), torch.float32),
                            "claim": ((N,), torch.int64)}, dev)
    for k in ("memory", "memory_ts", "mailbox", "mailbox_ts", "claim"):
        arena[k].zero_()
    tab = {k: arena.peer_table(k) for k in ("memory", "memory_ts", "mailbox", "mailbox_ts", "claim")}
    owner = (torch.arange(N, device=dev) % world).int()  # hash partition
    b = _ctdg_batch(N, events, D, rank, dev)
    efeat = torch.randn(events * world, E, device=dev)
    torch.cuda.synchronize()
    arena.barrier_host()
    flags = torch.zeros(32, dtype=torch.int64, device=dev)  # wait passes at epoch 0: claims only
    epoch = torch.zeros(1, dtype=torch.int64, device=dev)
    C.tgn_peer_wait_claim(flags, rank, world, epoch, 1_000_000, b["roots"], b["n_roots"], b["win"], b["ev_eid"],
                          b["ev_ts"], owner, tab["claim"])
    torch.cuda.synchronize()
    dist.barrier()  # every claim posted before the first push reads the winners

    def fused():
        C.tgn_peer_push(b["roots"], b["n_roots"], b["mem_new"], b["ts_max"], owner, tab["memory"],
                        tab["memory_ts"], None, 0.0, rank, b["win"], b["src_idx"], b["dst_idx"], b["ev_eid"],
                        b["ev_ts"], b["mem_prev"], efeat, E, tab["claim"], tab["mailbox"], tab["mailbox_ts"])

    # NCCL form: per root [memory row | ts | mail slot | mail ts] to its owner
    R = b["R"]
    own = owner[b["roots"]].long()
    order = torch.argsort(own)
    send_counts = torch.bincount(own, minlength=world)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts)
    sc, rcn = send_counts.tolist(), recv_counts.tolist()
    recv_ids = torch.empty(int(sum(rcn)), dtype=torch.long, device=dev)
    dist.all_to_all_single(recv_ids, b["roots"][order], output_split_sizes=rcn, input_split_sizes=sc)
    last = torch.maximum(b["win"][:R], b["win"][R:]).long().clamp(min=0)  # a root's latest event
    is_src = b["win"][:R].long() >= b["win"][R:].long()
    self_r = torch.where(is_src, b["src_idx"][last].long(), b["dst_idx"][last].long())
    other_r = torch.where(is_src, b["dst_idx"][last].long(), b["src_idx"][last].long())
    W1 = D + 1 + SW + 1
    recv = torch.empty(int(sum(rcn)), W1, device=dev)
    mem, mts = arena["memory"], arena["memory_ts"]
    mail, mail_ts = arena["mailbox"], arena["mailbox_ts"]

    def nccl():
        payload = torch.cat([b["mem_new"], b["ts_max"].expand(R, 1), b["mem_prev"][self_r], b["mem_prev"][other_r],
                             efeat[b["ev_eid"][last]], b["ev_ts"][last].view(-1, 1)], dim=1)[order]
        dist.all_to_all_single(recv, payload, output_split_sizes=rcn, input_split_sizes=sc)
        mem.index_copy_(0, recv_ids, recv[:, :D])
        mts.index_copy_(0, recv_ids, recv[:, D])
        mail.index_copy_(0, recv_ids, recv[:, D + 1:D + 1 + SW])
        mail_ts.index_copy_(0, recv_ids, recv[:, -1])

    fused_ms = _time(fused, iters, warmup)
    nccl_ms = _time(nccl, iters, warmup)
    remote = int((own != rank).sum())
    # per remote root: memory row + ts, mail slot + ts (at most: only claim winners write mail)
    nvl = remote * (D + 1 + SW + 1) * 4.0
    # local: new rows and previous rows read, edge-feature rows read, own roots' rows written
    hbm = R * (2 * D + E) * 4.0 + (R - remote) * (D + 1 + SW + 1) * 4.0
    r = _report("writeback", {"nodes": N, "events_per_rank": events, "roots_per_rank": R,
                              "remote_roots_per_rank": remote, "D": D, "E": E}, fused_ms, nccl_ms, nvl, hbm, world)
    arena.barrier_host()
    return r


def bench_remote_fetch(N: int, events: int, k: int, D: int, E: int, T: int, Do: int, iters: int, warmup: int,
                       C) -> dict:
    """Fused path #1: the attention projections of one CTDG step with node memory
    sharded over the ranks (``tgn_attn_proj`` with a peer descriptor: the operand
    producer reads each root's and each neighbour's memory row from its owner's
    table over NVLink while it packs the tcgen05 operand), against the NCCL form:
    the remote rows requested once per step with ``all_to_all_single`` into a
    local replica, then the same projections on the local table."""
    from starry_unigraph.parallel.symmetric import SymmetricArena

    world, rank = dist.get_world_size(), dist.get_rank()
    dev = torch.device("cuda", torch.cuda.current_device())
    arena = SymmetricArena({"memory": ((N, D), torch.float32)}, dev)
    owner = (torch.arange(N, device=dev) % world).int()
    g = torch.Generator(device=dev).manual_seed(99)
    full = torch.randn(N, D, device=dev, generator=g)  # the same values on every rank
    arena["memory"].copy_(torch.where((owner == rank).view(-1, 1), full, torch.zeros_like(full)))
    table = arena.peer_table("memory")
    b = _ctdg_batch(N, events, D, rank, dev)
    R = b["R"]
    gh = torch.Generator(device=dev).manual_seed(7 + rank)
    nbr = torch.randint(0, N, (R * k,), device=dev, generator=gh)
    nbr_eid = torch.randint(0, events * world, (R * k,), device=dev, generator=gh)
    nbr_dt = torch.rand(R * k, device=dev, generator=gh) * 1e4
    nbr_cnt = torch.full((R,), k, dtype=torch.int32, device=dev)
    efeat = torch.randn(events * world, E, device=dev)
    te_w, te_b = torch.randn(T, device=dev), torch.randn(T, device=dev)
    wq, bq = torch.randn(Do, D + T, device=dev) * 0.1, torch.randn(Do, device=dev)
    wk, bk = torch.randn(Do, D + E + T, device=dev) * 0.1, torch.randn(Do, device=dev)
    wv, bv = torch.randn(Do, D + E + T, device=dev) * 0.1, torch.randn(Do, device=dev)
    Q, KV = torch.zeros(R, Do, device=dev), torch.zeros(R * k, 2 * Do, device=dev)
    stamp = torch.zeros(N, dtype=torch.int32, device=dev)  # no fresh rows this step
    node2root = torch.zeros(N, dtype=torch.int32, device=dev)
    step = torch.full((1,), 7, dtype=torch.int64, device=dev)
    mem_new = torch.zeros(R, D, device=dev)
    desc = torch.tensor([table.data_ptr(), 0, owner.data_ptr(), stamp.data_ptr(), node2root.data_ptr(),
                         step.data_ptr(), mem_new.data_ptr()], dtype=torch.int64)
    torch.cuda.synchronize()
    arena.barrier_host()

    def fused():
        C.tgn_attn_proj(arena["memory"], b["roots"], b["n_roots"], nbr, nbr_eid, nbr_dt, nbr_cnt, efeat, E, te_w,
                        te_b, wq, bq, wk, bk, wv, bv, Q, KV, desc)

    # NCCL form: unique remote rows (roots and neighbours) grouped by owner
    need = torch.unique(torch.cat([b["roots"], nbr]))
    need = need[owner[need] != rank]
    need = need[torch.argsort(owner[need].long(), stable=True)]
    req_counts = torch.bincount(owner[need].long(), minlength=world)
    ask_counts = torch.empty_like(req_counts)
    dist.all_to_all_single(ask_counts, req_counts)
    rc, ac = req_counts.tolist(), ask_counts.tolist()
    asked = torch.empty(int(sum(ac)), dtype=torch.long, device=dev)
    dist.all_to_all_single(asked, need, output_split_sizes=ac, input_split_sizes=rc)
    replica = arena["memory"].clone()
    got = torch.empty(need.numel(), D, device=dev)
    Q2, KV2 = torch.zeros_like(Q), torch.zeros_like(KV)

    def nccl():
        dist.all_to_all_single(got, arena["memory"].index_select(0, asked), output_split_sizes=rc,
                               input_split_sizes=ac)
        replica.index_copy_(0, need, got)
        C.tgn_attn_proj(replica, b["roots"], b["n_roots"], nbr, nbr_eid, nbr_dt, nbr_cnt, efeat, E, te_w, te_b,
                        wq, bq, wk, bk, wv, bv, Q2, KV2, None)

    fused(), nccl()
    torch.cuda.synchronize()
    err = max(float((Q - Q2).abs().max()), float((KV - KV2).abs().max()))
    fused_ms = _time(fused, iters, warmup)
    nccl_ms = _time(nccl, iters, warmup)
    remote_reads = int((owner[nbr] != rank).sum()) + int((owner[b["roots"]] != rank).sum())
    nvl = remote_reads * D * 4.0  # every remote row read crosses NVLink once per use
    # local: own rows read, edge-feature rows, outputs Q and KV written
    hbm = ((R * (k + 1) - remote_reads) * D + R * k * E + R * Do + R * k * 2 * Do) * 4.0
    r = _report("remote_fetch", {"nodes": N, "roots_per_rank": R, "neighbours": k, "D": D, "E": E, "T": T,
                                 "Do": Do, "remote_row_reads_per_rank": remote_reads,
                                 "unique_remote_rows_per_rank": int(need.numel())},
                fused_ms, nccl_ms, nvl, hbm, world)
    r["max_abs_diff_vs_nccl"] = err
    arena.barrier_host()
    return r


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--paths", default="allreduce_adam,halo_gather,writeback,remote_fetch")
    args = ap.parse_args()
    if not torch.cuda.is_available():
        print("bench_fused.py: the fused NVLink paths need CUDA devices and none is visible here", file=sys.stderr)
        sys.exit(2)
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    from starry_unigraph.ops import cuda_ext

    C = cuda_ext()
    out = []
    paths = args.paths.split(",")
    if "allreduce_adam" in paths:
        for n in (262_144, 4_194_304, 33_554_432):
            out.append(bench_allreduce_adam(n, args.iters, args.warmup, C))
    if "halo_gather" in paths:
        out.append(bench_halo_gather(200_000, 2_000_000, 64, args.iters, args.warmup, C))
    # the TGN headline shape: 1,140,149 nodes, 600 events per rank, memory 100, edge features 16
    if "writeback" in paths:
        out.append(bench_writeback(1_140_149, 600, 100, 16, args.iters, args.warmup, C))
    if "remote_fetch" in paths:
        out.append(bench_remote_fetch(1_140_149, 600, 10, 100, 16, 100, 100, args.iters, args.warmup, C))
    if dist.get_rank() == 0:
        for r in out:
            print(json.dumps(r), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
