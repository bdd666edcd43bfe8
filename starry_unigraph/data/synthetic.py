"""Synthetic event streams and snapshot sequences of the benchmark shapes.

* ``zipf_event_stream``: CTDG streams with Zipf-distributed endpoints
  (bipartite or unipartite), a fraction of repeated interactions, sorted
  uniform timestamps and N(0, 1) edge features.
* ``chung_lu_snapshots`` / ``rmat_snapshots``: DTDG snapshot sequences over a
  fixed node set with edge churn between consecutive snapshots.

Everything is generated from a seed with numpy; no network or external data.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import numpy as np
import torch


def _zipf_sampler(n: int, s: float, rng: np.random.Generator, size: int) -> np.ndarray:
    """Draw ``size`` ranks in [0, n) with P(rank k) proportional to (k+1)^-s."""
    w = np.power(np.arange(1, n + 1, dtype=np.float64), -s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    u = rng.random(size)
    return np.minimum(np.searchsorted(cdf, u, side="right"), n - 1).astype(np.int64)


def zipf_event_stream(
    num_src: int,
    num_dst: int,
    num_events: int,
    *,
    s_src: float,
    s_dst: float,
    bipartite: bool,
    repeat_frac: float = 0.0,
    t_max: float = 1.0,
    edge_dim: int = 16,
    edge_dtype: torch.dtype = torch.float32,
    seed: int = 0,
) -> dict[str, Any]:
    rng = np.random.default_rng(seed)
    n_nodes = num_src + num_dst if bipartite else num_src
    perm_src = rng.permutation(num_src)
    src = perm_src[_zipf_sampler(num_src, s_src, rng, num_events)]
    if bipartite:
        perm_dst = rng.permutation(num_dst)
        dst = num_src + perm_dst[_zipf_sampler(num_dst, s_dst, rng, num_events)]
    else:
        perm_dst = rng.permutation(num_src)
        dst = perm_dst[_zipf_sampler(num_src, s_dst, rng, num_events)]
        self_loop = dst == src
        dst[self_loop] = (dst[self_loop] + 1) % num_src
    if repeat_frac > 0:
        rep = np.nonzero(rng.random(num_events) < repeat_frac)[0]
        rep = rep[rep > 0]
        prev = (rng.random(rep.size) * rep).astype(np.int64)
        src[rep] = src[prev]
        dst[rep] = dst[prev]
    ts = np.sort(rng.random(num_events) * t_max).astype(np.float32)
    gen = torch.Generator().manual_seed(seed + 1)
    edge_feat = torch.randn(num_events, edge_dim, generator=gen).to(edge_dtype)
    return {
        "src": torch.from_numpy(src),
        "dst": torch.from_numpy(dst),
        "ts": torch.from_numpy(ts),
        "edge_feat": edge_feat,
        "num_nodes": int(n_nodes),
    }


# Presets named after the benchmark configurations.
CTDG_PRESETS: dict[str, dict[str, Any]] = {
    # 9,227 nodes (8,227 src + 1,000 dst), 157,474 events, Zipf(1.1), 172-dim features
    "tgn_cpu": dict(num_src=8227, num_dst=1000, num_events=157474, s_src=1.1, s_dst=1.1, bipartite=True,
                    t_max=2.7e6, edge_dim=172),
    # 1,140,149 nodes, 7,833,140 events, Zipf(1.2), 20% repeats, 16-dim features
    "tgn_large": dict(num_src=1140149, num_dst=0, num_events=7833140, s_src=1.2, s_dst=1.2, bipartite=False,
                      repeat_frac=0.2, t_max=1.9e8, edge_dim=16),
    # 10M users + 1M items, 200M events, users Zipf(1.0), items Zipf(1.3), 32-dim bf16 features
    "jodie_large": dict(num_src=10_000_000, num_dst=1_000_000, num_events=200_000_000, s_src=1.0, s_dst=1.3,
                        bipartite=True, t_max=3e7, edge_dim=32, edge_dtype=torch.bfloat16),
}


def ctdg_preset(name: str, *, num_events: int | None = None, seed: int = 0) -> dict[str, Any]:
    spec = dict(CTDG_PRESETS[name])
    if num_events is not None:
        spec["num_events"] = int(num_events)
    return zipf_event_stream(**spec, seed=seed)


@dataclass
class SnapshotSpec:
    num_nodes: int
    num_snapshots: int
    edges_per_snapshot: int
    churn: float
    feat_dim: int
    generator: str = "chung_lu"   # chung_lu | rmat
    degree_exponent: float = 2.1
    rmat: tuple[float, float, float] = (0.57, 0.19, 0.19)
    label: str = "regression"     # regression | binary
    seed: int = 0


class _InverseCDF:
    """Draws indices i in [0, n) with probability p_i by inverse transform, with
    a bucket table in place of a binary search per sample: bucket j of M equal
    slices of [0, 1) stores the first index whose cumulative mass exceeds j / M,
    and a sample walks forward from its bucket's index (a few steps at most when
    M exceeds the number of indices with non-negligible mass per slice). Gives
    the same indices as ``searchsorted(cdf, u, side="right")``."""

    def __init__(self, w: np.ndarray, buckets: int = 1 << 22):
        cdf = np.cumsum(w, dtype=np.float64)
        cdf /= cdf[-1]
        self.cdf = cdf
        self.m = int(buckets)
        self.table = np.searchsorted(cdf, np.arange(self.m, dtype=np.float64) / self.m, side="right")

    def __call__(self, u: np.ndarray) -> np.ndarray:
        idx = self.table[np.minimum((u * self.m).astype(np.int64), self.m - 1)]
        n = self.cdf.size
        todo = np.arange(u.size)
        while todo.size:
            i = idx[todo]
            adv = (i < n - 1) & (self.cdf[np.minimum(i, n - 1)] <= u[todo])
            todo = todo[adv]
            idx[todo] += 1
        return np.minimum(idx, n - 1)


_CDF_CACHE: dict[tuple, _InverseCDF] = {}


def _chung_lu_edges(n: int, m: int, gamma: float, rng: np.random.Generator, perm: np.ndarray) -> np.ndarray:
    # expected degrees w_i ~ i^(-1/(gamma-1)); endpoints drawn proportionally to w
    key = (int(n), float(gamma))
    if key not in _CDF_CACHE:
        _CDF_CACHE.clear()
        _CDF_CACHE[key] = _InverseCDF(np.power(np.arange(1, n + 1, dtype=np.float64), -1.0 / (gamma - 1.0)))
    u = rng.random(2 * m)
    return perm[_CDF_CACHE[key](u).reshape(2, m)]


def _rmat_edges(n: int, m: int, abc: tuple[float, float, float], rng: np.random.Generator) -> np.ndarray:
    a, b, c = abc
    bits = int(np.ceil(np.log2(max(2, n))))
    src = np.zeros(m, dtype=np.int64)
    dst = np.zeros(m, dtype=np.int64)
    for _ in range(bits):
        r = rng.random(m)
        q_b = (r >= a) & (r < a + b)
        q_c = (r >= a + b) & (r < a + b + c)
        q_d = r >= a + b + c
        src = (src << 1) | (q_c | q_d)
        dst = (dst << 1) | (q_b | q_d)
    return np.stack([src % n, dst % n])


def snapshot_sequence(spec: SnapshotSpec) -> list[dict[str, Any]]:
    """Snapshots as dicts {edge_index [2, E], edge_weight [E], x [N, F], y [N] or None}."""
    rng = np.random.default_rng(spec.seed)
    perm = rng.permutation(spec.num_nodes)
    gen = torch.Generator().manual_seed(spec.seed + 7)

    def fresh(m: int) -> np.ndarray:
        if spec.generator == "rmat":
            return _rmat_edges(spec.num_nodes, m, spec.rmat, rng)
        return _chung_lu_edges(spec.num_nodes, m, spec.degree_exponent, rng, perm)

    edges = fresh(spec.edges_per_snapshot)
    out: list[dict[str, Any]] = []
    for t in range(spec.num_snapshots):
        if t > 0 and spec.churn > 0:
            k = int(round(spec.churn * edges.shape[1]))
            drop = rng.choice(edges.shape[1], size=k, replace=False)
            edges = edges.copy()
            edges[:, drop] = fresh(k)
        ei = torch.from_numpy(np.ascontiguousarray(edges)).long()
        x = torch.randn(spec.num_nodes, spec.feat_dim, generator=gen)
        if spec.label == "binary":
            y = torch.randint(0, 2, (spec.num_nodes,), generator=gen).float()
        else:
            y = torch.randn(spec.num_nodes, generator=gen)
        out.append({"edge_index": ei, "edge_weight": torch.ones(ei.size(1)), "x": x, "y": y})
    return out


DTDG_PRESETS: dict[str, SnapshotSpec] = {
    "mpnn_lstm_large": SnapshotSpec(num_nodes=200_000, num_snapshots=128, edges_per_snapshot=2_000_000, churn=0.3,
                                    feat_dim=64, generator="chung_lu", degree_exponent=2.1),
    "egcn_large": SnapshotSpec(num_nodes=2_000_000, num_snapshots=32, edges_per_snapshot=20_000_000, churn=0.1,
                               feat_dim=128, generator="rmat", label="binary"),
}
