"""Single-GPU timings of the DTDG hot kernels in isolation.

    python bench_kernels.py spmm     # CSR aggregation, 200k rows x 2M edges, F = 64 (edge-stream and item kernels)
    python bench_kernels.py lstm     # fused LSTM cell forward and backward, 200k rows, hidden 64
    python bench_kernels.py linear   # GCN linear forward / input gradient, 200k rows, 64 -> 64 and 128 -> 256

Each case prints one JSON line of device times (CUDA events on the current
stream, 5 warm-up calls, mean of 20, synchronised on both sides). The inputs
are larger than the 126 MB L2 except the SpMM feature matrix (51 MB), which a
real aggregation also keeps resident. The SpMM case also times cuSPARSE
(``torch.sparse_csr_tensor @ x``) on the same matrix, a uniform-degree graph
and a graph with sequential columns (every gather next to the previous one).
"""
from __future__ import annotations

import json
import sys

import torch

from starry_unigraph.ops import cuda_ext


def _time(fn, iters: int = 20, warmup: int = 5) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1000.0


def spmm() -> dict:
    C = cuda_ext()
    dev = "cuda"
    n, m, F = 200_000, 2_000_000, 64
    torch.manual_seed(1)
    g = torch.Generator().manual_seed(1)
    deg = torch.distributions.Pareto(torch.tensor(1.0), torch.tensor(1.5)).sample((n,)).clamp(max=50_000)
    deg = (deg / deg.sum() * m).round().long()
    rowptr = torch.zeros(n + 1, dtype=torch.long)
    rowptr[1:] = deg.cumsum(0)
    nnz = int(rowptr[-1])
    col = torch.randint(0, n, (nnz,), dtype=torch.int32, generator=g)
    val = torch.rand(nnz, generator=g)
    x = torch.randn(n, F, device=dev)
    rp, cl, vl = rowptr.to(dev), col.to(dev), val.to(dev)
    out = torch.empty(n, F, device=dev)
    t = _time(lambda: C.spmm_csr(rp, cl, vl, x, n, out, False))
    from starry_unigraph.data.partition import spmm_plan

    plan = spmm_plan(rp)
    t_items = _time(lambda: C.spmm_csr(rp, cl, vl, x, n, out, False, plan))
    A = torch.sparse_csr_tensor(rp, cl.long(), vl, size=(n, n))
    t_cusparse = _time(lambda: A @ x)
    rp2 = torch.arange(0, n + 1, device=dev, dtype=torch.long) * (m // n)
    cl2 = torch.randint(0, n, (m,), dtype=torch.int32, device=dev)
    vl2 = torch.rand(m, device=dev)
    t_uniform = _time(lambda: C.spmm_csr(rp2, cl2, vl2, x, n, out, False))
    cl3 = torch.arange(m, device=dev, dtype=torch.int32) % n
    t_seq = _time(lambda: C.spmm_csr(rp2, cl3, vl2, x, n, out, False))
    return {"case": "spmm", "rows": n, "nnz": nnz, "F": F, "max_row": int(deg.max()), "spmm_us": round(t, 1),
            "items_us": round(t_items, 1),
            "cusparse_us": round(t_cusparse, 1), "uniform_rows_us": round(t_uniform, 1),
            "sequential_cols_us": round(t_seq, 1)}


def lstm() -> dict:
    C = cuda_ext()
    dev = "cuda"
    rows, IN, H = 200_000, 64, 64
    torch.manual_seed(0)
    x = torch.randn(rows, IN, device=dev)
    h, c = torch.randn(rows, H, device=dev), torch.randn(rows, H, device=dev)
    w = [torch.randn(H, IN + H, device=dev) * 0.1 for _ in range(4)]
    b = [torch.randn(H, device=dev) * 0.1 for _ in range(4)]
    fwd = lambda: C.lstm_fwd(x, h, c, w[0], b[0], w[1], b[1], w[2], b[2], w[3], b[3], True)  # noqa: E731
    t_fwd = _time(fwd)
    _, cn, gates = fwd()
    dh, dc = torch.randn(rows, H, device=dev), torch.randn(rows, H, device=dev)
    gw = [torch.zeros(H, IN + H, device=dev) for _ in range(4)]
    gb = [torch.zeros(H, device=dev) for _ in range(4)]
    t_bwd = _time(lambda: C.lstm_bwd(x, h, c, cn, gates, dh, dc, w[0], w[1], w[2], w[3], gw[0], gb[0], gw[1], gb[1],
                                     gw[2], gb[2], gw[3], gb[3]))
    return {"case": "lstm", "rows": rows, "in": IN, "hidden": H, "fwd_us": round(t_fwd, 1), "bwd_us": round(t_bwd, 1)}


def linear() -> dict:
    """Packed tcgen05 linear with the per-row store epilogue against the TMA-store
    epilogue (threshold switched per run); the memory roofline is the fp32 input
    read once plus the fp32 output written once at the measured copy bandwidth."""
    C = cuda_ext()
    rows = 200_000
    out = {"case": "linear", "rows": rows}
    old = C.tma_store_min_rows()
    try:
        for K, N in ((64, 64), (128, 256)):
            x = torch.randn(rows, K, device="cuda")
            w = torch.randn(N, K, device="cuda") / K ** 0.5
            gy = torch.randn(rows, N, device="cuda")
            for name, thr in (("direct", -1), ("tma", 0)):
                C.set_tma_store_min_rows(thr)
                out[f"fwd_{K}x{N}_{name}_us"] = round(_time(lambda: C.linear_fwd(x, w, None, 0)), 1)
                out[f"dgrad_{K}x{N}_{name}_us"] = round(_time(lambda: C.linear_dgrad(gy, w)), 1)
            out[f"fwd_{K}x{N}_bytes"] = rows * (K + N) * 4
    finally:
        C.set_tma_store_min_rows(old)
    return out


if __name__ == "__main__":
    if not torch.cuda.is_available():
        print("bench_kernels.py: the kernels run on a CUDA device and none is visible here", file=sys.stderr)
        sys.exit(2)
    cases = {"spmm": spmm, "lstm": lstm, "linear": linear}
    for name in (sys.argv[1:] or list(cases)):
        print(json.dumps(cases[name]()), flush=True)
