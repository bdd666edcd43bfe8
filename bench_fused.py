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
        return C.spmm_csr(csr["rowptr"], csr["col"], csr["val"], ext, n_local, None, False)

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


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--paths", default="allreduce_adam,halo_gather")
    args = ap.parse_args()
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
    if dist.get_rank() == 0:
        for r in out:
            print(json.dumps(r), flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
