"""DTDG data preparation: node partitioning, per-snapshot blocks, Flare export
(reference backends/dtdg/dtdg_prepare.py:45-537).

* ``apply_partition``: METIS through pymetis when installed; otherwise the
  native streaming partitioner of ``starry_unigraph._native`` (balancing a
  vertex weight with ``preprocess.partition_edge_share`` of it on edges; linear
  deterministic greedy with a balance cap over the symmetrised lifetime graph,
  followed by label-propagation refinement); random assignment only when
  neither is available (the reference's fallback).
* ``_build_snapshot_blocks``: global symmetric GCN normalisation
  w / (sqrt(in_deg_w[dst]) * sqrt(out_deg_w[src])) then ``Route.from_graph``.
* ``build_flare_partition_data_list``: per-partition ``PartitionData`` with node
  features (source rows incl. halo), labels (destination rows), weights, norms,
  routes, the chunk index ``c`` (a second partitioning of each partition's
  induced lifetime graph into ``preprocess.cluster.num_per_partition`` chunks)
  and ``partition_id``.
"""
from __future__ import annotations

from typing import Any

import torch

from starry_unigraph.data.partition import EID, NID, PartitionData, TensorData

from .runtime.route import Route
from .types import SnapshotRoutePlan

try:  # optional, like in the reference
    import pymetis  # type: ignore
except Exception:  # pragma: no cover
    pymetis = None


def _as_int(value: Any, default: int) -> int:
    try:
        return int(value)
    except (TypeError, ValueError):
        return default


def _merge_snapshot_edges(snapshots: list[dict[str, Any]]) -> torch.Tensor:
    parts = [s["edge_index"].long() for s in snapshots if s["edge_index"].numel() > 0]
    return torch.cat(parts, dim=1) if parts else torch.zeros((2, 0), dtype=torch.long)


def apply_partition(edge_index: torch.Tensor, num_nodes: int, num_parts: int, seed: int = 0,
                    edge_share: float = 0.0) -> torch.Tensor:
    """Part of every node. Native partitioner: parts balance a vertex weight in
    which `edge_share` of the total goes to edge endpoints and the rest to nodes
    (0: node counts)."""
    num_nodes, num_parts = max(0, int(num_nodes)), max(1, int(num_parts))
    if num_nodes == 0:
        return torch.zeros(0, dtype=torch.long)
    if num_parts <= 1:
        return torch.zeros(num_nodes, dtype=torch.long)
    src, dst = edge_index[0].long().cpu(), edge_index[1].long().cpu()
    if pymetis is not None:
        import numpy as np
        import scipy.sparse as sp

        adj = sp.csr_matrix((np.ones(src.numel(), dtype=np.int32), (src.numpy(), dst.numpy())),
                            shape=(num_nodes, num_nodes))
        adj = (adj + adj.T).astype(np.int32)
        try:
            _, membership = pymetis.part_graph(nparts=num_parts, xadj=adj.indptr.astype(np.int32),
                                               adjncy=adj.indices.astype(np.int32))
            return torch.tensor(membership, dtype=torch.long)
        except Exception as exc:
            print(f"[Partition] pymetis failed: {exc}; using the native partitioner")
    from starry_unigraph.ops import native_ext

    nat = native_ext()
    if nat is not None:
        return nat.partition_graph(src.contiguous(), dst.contiguous(), num_nodes, num_parts, 1.03, 3, seed,
                                   float(edge_share)).long()
    print("[Partition] pymetis and the native partitioner unavailable; random partition")
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, num_parts, (num_nodes,), generator=g)


def build_dtdg_partitions(graph_data: Any, num_parts: int, algo: str, config: dict[str, Any]) -> dict[str, Any]:
    num_nodes = int(graph_data["num_nodes"])
    merged = _merge_snapshot_edges(list(graph_data.get("dataset", [])))
    algo_l = str(algo).lower()
    if algo_l in ("random",):
        node_parts = torch.randint(0, max(1, num_parts), (num_nodes,), generator=torch.Generator().manual_seed(0))
    elif algo_l in ("round_robin", "hash"):
        node_parts = torch.arange(num_nodes) % max(1, num_parts)
    else:
        share = float(config.get("preprocess", {}).get("partition_edge_share", 0.0))
        node_parts = apply_partition(merged, num_nodes, max(1, num_parts), edge_share=share)
    parts = [{"partition_id": p, "node_ids": torch.nonzero(node_parts == p).view(-1),
              "num_nodes": int((node_parts == p).sum())} for p in range(max(1, num_parts))]
    return {"algo": algo, "num_parts": max(1, num_parts), "node_parts": node_parts, "parts": parts,
            "graph_stats": {"num_nodes": num_nodes, "num_edges": int(graph_data["num_edges"]),
                            "num_snapshots": int(graph_data["num_snapshots"]),
                            "window_size": _as_int(config.get("model", {}).get("window", {}).get("size"), 1)}}


def _compute_degrees(edge_index: torch.Tensor, w: torch.Tensor, num_nodes: int):
    if edge_index.numel() == 0:
        z = torch.zeros(num_nodes)
        return z, z
    return (torch.bincount(edge_index[1], weights=w, minlength=num_nodes).float(),
            torch.bincount(edge_index[0], weights=w, minlength=num_nodes).float())


def _build_snapshot_blocks(snapshot_index: int, snapshot: dict[str, Any], node_parts: torch.Tensor, num_parts: int,
                           num_nodes: int, route_plan: SnapshotRoutePlan):
    ei = snapshot["edge_index"].long()
    w = snapshot["edge_weight"].float()
    x = snapshot["x"]
    y = snapshot.get("y")
    in_deg, out_deg = _compute_degrees(ei, w, num_nodes)
    if ei.numel():
        norm = (w / (torch.sqrt(in_deg.clamp_min(1e-12))[ei[1]] * torch.sqrt(out_deg.clamp_min(1e-12))[ei[0]]))
        norm = norm.nan_to_num(0.0)
    else:
        norm = torch.zeros(0)
    blocks = Route.from_graph(node_parts, ei, num_parts=num_parts)
    for pid, blk in enumerate(blocks):
        s_ids, d_ids, e_ids = blk.srcdata[NID], blk.dstdata[NID], blk.edata[EID]
        blk.srcdata["x"] = x[s_ids] if s_ids.numel() else torch.zeros((0, x.size(-1)), dtype=x.dtype)
        blk.dstdata["y"] = y[d_ids] if (y is not None and d_ids.numel()) else torch.zeros(d_ids.numel())
        blk.edata["w"] = w[e_ids] if e_ids.numel() else torch.zeros(0)
        blk.edata["gcn_norm"] = norm[e_ids] if e_ids.numel() else torch.zeros(0)
        blk.graph_meta = {"snapshot_index": snapshot_index, "partition_id": pid, "route_plan": route_plan.describe(),
                          "num_nodes": num_nodes, "route": blk.route.describe()}
    return blocks


def _induced_local_edges(merged: torch.Tensor, local_nodes: torch.Tensor, num_nodes: int) -> torch.Tensor:
    if local_nodes.numel() == 0 or merged.numel() == 0:
        return torch.zeros((2, 0), dtype=torch.long)
    loc = torch.full((num_nodes,), -1, dtype=torch.long)
    loc[local_nodes] = torch.arange(local_nodes.numel())
    s, d = loc[merged[0]], loc[merged[1]]
    keep = (s >= 0) & (d >= 0)
    return torch.stack([s[keep], d[keep]])


def build_flare_partition_data_list(raw_dataset: dict[str, Any], partition_result: dict[str, Any],
                                    route_plan: SnapshotRoutePlan, config: dict[str, Any]) -> list[PartitionData]:
    dataset = list(raw_dataset["dataset"])
    node_parts = partition_result["node_parts"].long()
    num_parts = int(partition_result["num_parts"])
    num_nodes = int(raw_dataset["num_nodes"])
    chunks = max(1, _as_int(config.get("preprocess", {}).get("cluster", {}).get("num_per_partition"), 1))
    merged = _merge_snapshot_edges(dataset)
    per_part: list[list] = [[] for _ in range(num_parts)]
    for si, snap in enumerate(dataset):
        for pid, blk in enumerate(_build_snapshot_blocks(si, snap, node_parts, num_parts, num_nodes, route_plan)):
            per_part[pid].append(blk)
    out = []
    for pid in range(num_parts):
        local = torch.nonzero(node_parts == pid).view(-1)
        pdata = PartitionData.from_blocks(per_part[pid])
        n_chunks = min(chunks, max(1, int(local.numel())))
        cidx = apply_partition(_induced_local_edges(merged, local, num_nodes), int(local.numel()), n_chunks, seed=pid)
        pdata.add_ndata("c", TensorData.from_tensors([cidx.clone() for _ in range(len(pdata))]))
        pdata.add_ndata("partition_id", TensorData.from_tensors(
            [torch.full((local.numel(),), pid, dtype=torch.long) for _ in range(len(pdata))]))
        out.append(pdata)
    return out


def normalize_snapshot_count(raw_dataset: dict[str, Any], snaps: int) -> dict[str, Any]:
    ds = list(raw_dataset.get("dataset", []))
    if not ds:
        return raw_dataset
    ds = ds[:snaps]
    while len(ds) < snaps:
        t = ds[-1]
        ds.append({"edge_index": t["edge_index"].clone(), "edge_weight": t["edge_weight"].clone(),
                   "x": t["x"].clone(), "y": None if t.get("y") is None else t["y"].clone()})
    return {**raw_dataset, "dataset": ds, "num_snapshots": len(ds),
            "num_life_edges": int(sum(int(d["edge_weight"].numel()) for d in ds))}
