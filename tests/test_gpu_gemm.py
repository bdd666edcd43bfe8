"""tcgen05 GEMM numerics against a plain fp32 PyTorch reference: bf16 operands
(kind::f16, relative tolerance ~1e-2) and tf32 operands (kind::tf32, relative
tolerance ~2e-3), fp32 accumulation either way."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from starry_unigraph.ops import cuda_ext

    return cuda_ext()


def _rel(a, b):
    return float((a - b).norm() / (b.norm() + 1e-12))


@pytest.mark.parametrize("M,K,N", [(1, 8, 16), (128, 64, 128), (300, 100, 100), (1000, 216, 200), (257, 33, 300),
                                   (4096, 128, 512), (130, 256, 600)])
def test_linear_fwd(M, K, N):
    C = _C()
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / K ** 0.5
    b = torch.randn(N, device="cuda")
    y = C.linear_fwd(x, w, b, 0)
    ref = x @ w.t() + b
    torch.cuda.synchronize()
    assert C.status_read(True) == 0
    assert _rel(y, ref) < 1.5e-2, _rel(y, ref)


@pytest.mark.parametrize("act", [1, 2, 3])
def test_linear_act(act):
    C = _C()
    x = torch.randn(200, 64, device="cuda")
    w = torch.randn(96, 64, device="cuda") / 8
    y = C.linear_fwd(x, w, None, act)
    z = x @ w.t()
    ref = {1: torch.relu, 2: torch.sigmoid, 3: torch.tanh}[act](z)
    assert _rel(y, ref) < 1.5e-2


@pytest.mark.parametrize("M,K,N", [(64, 16, 32), (1000, 100, 200), (3000, 216, 100)])
def test_linear_dgrad(M, K, N):
    C = _C()
    dy = torch.randn(M, N, device="cuda")
    w = torch.randn(N, K, device="cuda") / N ** 0.5
    dx = C.linear_dgrad(dy, w)
    assert _rel(dx, dy @ w) < 1.5e-2


@pytest.mark.parametrize("M,K,N", [(64, 16, 32), (1000, 100, 200), (12000, 216, 100)])
def test_linear_wgrad(M, K, N):
    C = _C()
    dy = torch.randn(M, N, device="cuda")
    x = torch.randn(M, K, device="cuda")
    dw = torch.zeros(N, K, device="cuda")
    db = torch.zeros(N, device="cuda")
    C.linear_wgrad(dy, x, dw, db)
    assert _rel(dw, dy.t() @ x) < 1.5e-2
    assert _rel(db, dy.sum(0)) < 1.5e-2


def test_adam_matches_torch():
    from starry_unigraph.ops.flat import FlatParams, FusedAdam

    torch.manual_seed(0)
    m1 = torch.nn.Linear(37, 11).cuda()
    m2 = torch.nn.Linear(37, 11).cuda()
    m2.load_state_dict(m1.state_dict())
    flat = FlatParams([m1], torch.device("cuda"))
    opt = FusedAdam(flat, lr=1e-2, weight_decay=0.01)
    ref = torch.optim.Adam(m2.parameters(), lr=1e-2, weight_decay=0.01)
    for _ in range(5):
        x = torch.randn(8, 37, device="cuda")
        flat.zero_grad()
        m1(x).pow(2).sum().backward()
        opt.step()
        ref.zero_grad()
        m2(x).pow(2).sum().backward()
        ref.step()
    for a, b in zip(m1.parameters(), m2.parameters()):
        assert torch.allclose(a, b, atol=1e-5, rtol=1e-4)


@pytest.fixture
def tf32():
    C = _C()
    C.set_gemm_precision(True)
    yield C
    C.set_gemm_precision(False)


def _fp32_ref(fn):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return fn()
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("M,K,N", [(1, 8, 16), (128, 64, 128), (300, 100, 100), (1000, 216, 200), (257, 33, 300),
                                   (4096, 128, 512)])
def test_linear_fwd_tf32(tf32, M, K, N):
    C = tf32
    torch.manual_seed(0)
    x = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / K ** 0.5
    b = torch.randn(N, device="cuda")
    y = C.linear_fwd(x, w, b, 0)
    ref = _fp32_ref(lambda: x @ w.t() + b)
    torch.cuda.synchronize()
    assert C.status_read(True) == 0
    assert _rel(y, ref) < 2e-3, _rel(y, ref)


@pytest.mark.parametrize("M,K,N", [(64, 16, 32), (1000, 100, 200), (3000, 216, 100)])
def test_linear_dgrad_wgrad_tf32(tf32, M, K, N):
    """The transposed operands (W^T of the data gradient, dY^T and X^T of the weight
    gradient) are transposed by the pack kernel into K-major tf32 images."""
    C = tf32
    torch.manual_seed(1)
    dy = torch.randn(M, N, device="cuda")
    w = torch.randn(N, K, device="cuda") / N ** 0.5
    x = torch.randn(M, K, device="cuda")
    dx = C.linear_dgrad(dy, w)
    assert _rel(dx, _fp32_ref(lambda: dy @ w)) < 2e-3
    dw = torch.zeros(N, K, device="cuda")
    db = torch.zeros(N, device="cuda")
    C.linear_wgrad(dy, x, dw, db)
    assert _rel(dw, _fp32_ref(lambda: dy.t() @ x)) < 2e-3
    assert _rel(db, dy.sum(0)) < 1e-3  # the bias gradient comes from a ones column of the tf32 GEMM


@pytest.fixture
def tma_rows():
    """Restores the TMA-store row threshold after a test that changes it."""
    C = _C()
    old = C.tma_store_min_rows()
    yield C
    C.set_tma_store_min_rows(old)


@pytest.mark.parametrize("M,K,N,act", [(2048, 64, 64, 0), (5000, 64, 100, 1), (20011, 128, 256, 0),
                                       (333, 96, 48, 3), (4099, 216, 130, 2)])
def test_linear_tma_store_matches_direct_stores(tma_rows, M, K, N, act):
    """The TMA-store epilogue (swizzled shared-memory boxes, tiled bulk stores)
    writes exactly what the per-row store epilogue writes, clipped to M x N."""
    C = tma_rows
    torch.manual_seed(1)
    x = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / K ** 0.5
    b = torch.randn(N, device="cuda")
    C.set_tma_store_min_rows(0)
    y_tma = C.linear_fwd(x, w, b, act)
    gx_tma = C.linear_dgrad(y_tma, w)
    C.set_tma_store_min_rows(-1)
    y_dir = C.linear_fwd(x, w, b, act)
    gx_dir = C.linear_dgrad(y_dir, w)
    torch.cuda.synchronize()
    assert C.status_read(True) == 0
    assert torch.equal(y_tma, y_dir)
    assert torch.equal(gx_tma, gx_dir)
    z = x @ w.t() + b
    ref = {0: z, 1: torch.relu(z), 2: torch.sigmoid(z), 3: torch.tanh(z)}[act]
    assert _rel(y_tma, ref) < 1.5e-2



@pytest.mark.parametrize("rows,IN,H,with_c", [(2500, 64, 64, True), (20011, 32, 48, False), (4096, 100, 32, True)])
def test_lstm_tma_store_matches_staged_stores(tma_rows, rows, IN, H, with_c):
    """The LSTM cell epilogue's TMA-store path (swizzled shared-memory boxes of
    the gates, c' and h') writes exactly what its staged-store path writes."""
    C = tma_rows
    torch.manual_seed(2)
    x = torch.randn(rows, IN, device="cuda")
    h = torch.randn(rows, H, device="cuda")
    c = torch.randn(rows, H, device="cuda") if with_c else None
    w = [torch.randn(H, IN + H, device="cuda") * 0.1 for _ in range(4)]
    b = [torch.randn(H, device="cuda") * 0.1 for _ in range(4)]
    args = (x, h, c, w[0], b[0], w[1], b[1], w[2], b[2], w[3], b[3], True)
    C.set_tma_store_min_rows(0)
    h1, c1, g1 = C.lstm_fwd(*args)
    C.set_tma_store_min_rows(-1)
    h2, c2, g2 = C.lstm_fwd(*args)
    torch.cuda.synchronize()
    assert C.status_read(True) == 0
    assert torch.equal(h1, h2) and torch.equal(c1, c2) and torch.equal(g1, g2)
    # and against the fp32 math of one nn.Linear per gate over [x || h]
    xh = torch.cat([x, h], 1)
    i, f, g, o = (xh @ w[k].t() + b[k] for k in range(4))
    cn = torch.sigmoid(f) * (c if with_c else 0) + torch.sigmoid(i) * torch.tanh(g)
    hn = torch.sigmoid(o) * torch.tanh(cn)
    assert _rel(c1, cn) < 2e-2 and _rel(h1, hn) < 2e-2


@pytest.mark.parametrize("M,K,N,ld", [(3000, 64, 64, 96), (500, 32, 64, 64), (5000, 128, 48, 128)])
def test_linear_fwd_into_row_strided_view(tma_rows, M, K, N, ld):
    """linear_fwd_into writes X W^T into the first N columns of a wider buffer's
    rows (a staging buffer with row stride ld) and leaves the other columns."""
    C = tma_rows
    x = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / K ** 0.5
    for thr in (0, -1):  # TMA-store and direct-store epilogues
        C.set_tma_store_min_rows(thr)
        buf = torch.full((M + 7, ld), 3.0, device="cuda")
        C.linear_fwd_into(x, w, None, 0, buf[:M, :N])
        torch.cuda.synchronize()
        assert C.status_read(True) == 0
        assert _rel(buf[:M, :N], x @ w.t()) < 1.5e-2
        assert torch.all(buf[:M, N:] == 3.0) and torch.all(buf[M:] == 3.0)


@pytest.mark.parametrize("M,K,N", [(3000, 64, 64), (777, 40, 100)])
def test_linear_grads_with_relu_mask_and_row_stride(M, K, N):
    """dY read through a row-strided view and masked by the forward output while
    it is packed: the data and weight gradients equal those of dY * (y > 0)."""
    C = _C()
    torch.manual_seed(3)
    x = torch.randn(M, K, device="cuda")
    w = torch.randn(N, K, device="cuda") / K ** 0.5
    y = torch.relu(x @ w.t())
    wide = torch.randn(M, N + 12, device="cuda")
    dy = wide[:, 4:4 + N]  # row stride N + 12
    ref = dy * (y > 0)
    dx = C.linear_dgrad(dy, w, y)
    dw, db = torch.zeros(N, K, device="cuda"), torch.zeros(N, device="cuda")
    C.linear_wgrad(dy, x, dw, db, y)
    torch.cuda.synchronize()
    assert C.status_read(True) == 0
    assert _rel(dx, ref @ w) < 1.5e-2
    assert _rel(dw, ref.t() @ x) < 1.5e-2
    assert _rel(db, ref.sum(0)) < 1.5e-2
