"""Multi-GPU CTDG training over NVLink (2 GPUs, torchrun). Skipped with fewer
than two GPUs."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
WORKER = ROOT / "tests" / "workers" / "ctdg_peer_worker.py"
DTDG_WORKER = ROOT / "tests" / "workers" / "dtdg_peer_worker.py"

need2 = pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                           reason="needs 2 GPUs")


def _run(out, nproc, *args, worker=WORKER, port=29613):
    env = dict(os.environ)
    env.setdefault("NCCL_NVLS_ENABLE", "0")
    if nproc == 1:
        cmd = [sys.executable, str(worker), "--out", str(out), *args]
    else:
        cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               f"--nproc-per-node={nproc}", "--master-addr", "127.0.0.1", "--master-port", str(port), str(worker),
               "--out", str(out), *args]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]


@need2
def test_owner0_run_matches_single_gpu(tmp_path):
    """All nodes and events on rank 0: the NVLink path (mem_new + write-back +
    mailbox claims) must reproduce the single-GPU step exactly (lr = 0)."""
    _run(tmp_path, 1, "--batch", "200", "--steps", "10", "--lr", "0", "--mode", "owner0")
    _run(tmp_path, 2, "--batch", "100", "--steps", "10", "--lr", "0", "--mode", "owner0")
    one = torch.load(tmp_path / "w1_r0.pt")
    two = torch.load(tmp_path / "w2_r0.pt")
    assert two["peer"] and not one["peer"]
    assert len(one["losses"]) == len(two["losses"]) == 10
    torch.testing.assert_close(torch.tensor(two["losses"]), torch.tensor(one["losses"]), rtol=1e-5, atol=1e-6)
    for k in ("memory", "memory_ts", "mailbox", "mailbox_ts"):
        torch.testing.assert_close(two[k], one[k], rtol=1e-5, atol=1e-6, msg=k)


@need2
@pytest.mark.parametrize("assign", ["balanced", "owner"])
def test_hash_partition_two_ranks_consistent(tmp_path, assign):
    _run(tmp_path, 2, "--batch", "100", "--steps", "12", "--mode", "hash", "--assign", assign)
    r0 = torch.load(tmp_path / "w2_r0.pt")
    r1 = torch.load(tmp_path / "w2_r1.pt")
    assert r0["peer"] and r1["peer"]
    if assign == "balanced":
        assert r0["sizes"] == r1["sizes"] == [100] * 12
    # the fused all-reduce sums in rank order on every rank: parameters stay bit-identical
    assert torch.equal(r0["params"], r1["params"])
    assert all(torch.isfinite(torch.tensor(r0["losses"] + r1["losses"])))
    # each node's row was written on its owner only
    owner = r0["owner"]
    touched = r0["memory_ts"] >= 0
    assert touched.any()
    assert not (r1["memory_ts"][owner == 0] >= 0).any()
    assert not (r0["memory_ts"][owner == 1] >= 0).any()


@need2
def test_async_sync_off_gives_the_same_steps(tmp_path):
    """ctdg.async_sync false makes each step wait for every peer's write-back; the
    overlapped default reads the same tables (the next step's remote reads wait
    for the peers' end signals either way), so the runs agree."""
    _run(tmp_path, 2, "--batch", "100", "--steps", "10", "--lr", "0", "--mode", "hash", port=29641)
    _run(tmp_path, 2, "--batch", "100", "--steps", "10", "--lr", "0", "--mode", "hash", "--sync", "--tag", "_sync",
         port=29642)
    for r in (0, 1):
        a = torch.load(tmp_path / f"w2_r{r}.pt")
        b = torch.load(tmp_path / f"w2_r{r}_sync.pt")
        torch.testing.assert_close(torch.tensor(b["losses"]), torch.tensor(a["losses"]), rtol=1e-6, atol=1e-7)
        for k in ("memory", "memory_ts", "mailbox", "mailbox_ts"):
            torch.testing.assert_close(b[k], a[k], rtol=1e-6, atol=1e-7, msg=k)


@need2
@pytest.mark.parametrize("decay", [False, True])
def test_dtdg_nvlink_halo_matches_nccl_route(tmp_path, decay):
    """MPNN-LSTM over 2 partitions: halo read from peer memory inside the
    aggregation + fused all-reduce/Adam must track the NCCL route + all-reduce;
    with decay, under a random chunk order (rows permuted per rank, published to
    the peers) and truncated older window slots."""
    extra = ["--decay"] if decay else []
    tag = "_decay" if decay else ""
    _run(tmp_path, 2, "--path", "nccl", *extra, worker=DTDG_WORKER, port=29631 + 4 * decay)
    _run(tmp_path, 2, "--path", "p2p", *extra, worker=DTDG_WORKER, port=29632 + 4 * decay)
    for r in (0, 1):
        a = torch.load(tmp_path / f"dtdg_p2p{tag}_r{r}.pt")
        b = torch.load(tmp_path / f"dtdg_nccl{tag}_r{r}.pt")
        assert a["halo"] is not None and b["halo"] is None
        torch.testing.assert_close(torch.tensor(a["losses"]), torch.tensor(b["losses"]), rtol=2e-3, atol=1e-5)
        torch.testing.assert_close(a["params"], b["params"], rtol=2e-3, atol=2e-5)
    # replicas identical under the fused all-reduce
    assert torch.equal(torch.load(tmp_path / f"dtdg_p2p{tag}_r0.pt")["params"],
                       torch.load(tmp_path / f"dtdg_p2p{tag}_r1.pt")["params"])
