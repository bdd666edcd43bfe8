"""The allocation-free C entry point su_lstm_cell_backward_noalloc against the
extension's lstm_bwd op on the same inputs, over two consecutive calls (the
second one reuses the static scratch array and accumulates into the same
gradient buffers). This file is collected last so that it also runs after the
rest of the suite has used the device."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    import starry_unigraph._C as C

    lib = ctypes.CDLL(C.__file__)
    f = lib.su_lstm_cell_backward_noalloc
    f.restype = ctypes.c_int
    f.argtypes = [ctypes.c_void_p] * 21 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    lib.su_noalloc_scratch_required.restype = ctypes.c_size_t
    lib.su_noalloc_scratch_required.argtypes = [ctypes.c_int] * 3
    lib.su_noalloc_scratch_capacity.restype = ctypes.c_size_t
    lib.su_noalloc_status.restype = ctypes.c_int
    lib.su_noalloc_status.argtypes = [ctypes.POINTER(ctypes.c_int)]
    lib.su_noalloc_status_reset.restype = ctypes.c_int
    lib.su_noalloc_strerror.restype = ctypes.c_char_p
    lib.su_noalloc_strerror.argtypes = [ctypes.c_int]
    return C, lib


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _case(rows, in_dim, H, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: torch.randn(*s, device="cuda", generator=g) * 0.5  # noqa: E731
    x, h, c = r(rows, in_dim), r(rows, H), r(rows, H)
    w = [r(H, in_dim + H).contiguous() for _ in range(4)]
    b = [r(H) for _ in range(4)]
    dh, dc = r(rows, H), r(rows, H)
    return x, h, c, w, b, dh, dc


def _call_noalloc(lib, x, h, c, cn, gates, dh, dc, w, gw, gb, rows, in_dim, H):
    dxh = torch.empty(rows, in_dim + H, device="cuda")
    dcp = torch.empty(rows, H, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.su_lstm_cell_backward_noalloc(
        _ptr(x), _ptr(h), _ptr(c), _ptr(cn), _ptr(gates), _ptr(dh), _ptr(dc), *[_ptr(t) for t in w],
        _ptr(gw[0]), _ptr(gb[0]), _ptr(gw[1]), _ptr(gb[1]), _ptr(gw[2]), _ptr(gb[2]), _ptr(gw[3]), _ptr(gb[3]),
        _ptr(dxh), _ptr(dcp), rows, in_dim, H, stream)
    return rc, dxh, dcp


@pytest.mark.parametrize("in_dim,H", [(20, 32), (64, 32), (24, 20)])
def test_noalloc_matches_lstm_bwd_on_two_calls(in_dim, H):
    """hidden = 20 exercises the padded hidden width (24) and the clipped output columns."""
    from starry_unigraph.ops import gemm_precision

    C, lib = _lib()
    rows = 1000
    assert lib.su_noalloc_status_reset() == 0
    gw_ref = [torch.zeros(H, in_dim + H, device="cuda") for _ in range(4)]
    gb_ref = [torch.zeros(H, device="cuda") for _ in range(4)]
    gw_na = [torch.zeros(H, in_dim + H, device="cuda") for _ in range(4)]
    gb_na = [torch.zeros(H, device="cuda") for _ in range(4)]
    for seed in (1, 2):
        x, h, c, w, b, dh, dc = _case(rows, in_dim, H, seed)
        with gemm_precision(False):  # the entry point runs bf16 operands; compare with the op in bf16
            _, cn, gates = C.lstm_fwd(x, h, c, w[0], b[0], w[1], b[1], w[2], b[2], w[3], b[3], True)
            dx_ref, dhp_ref, dcp_ref = C.lstm_bwd(x, h, c, cn, gates, dh, dc, w[0], w[1], w[2], w[3],
                                                  gw_ref[0], gb_ref[0], gw_ref[1], gb_ref[1], gw_ref[2],
                                                  gb_ref[2], gw_ref[3], gb_ref[3])
        rc, dxh, dcp = _call_noalloc(lib, x, h, c, cn, gates, dh, dc, w, gw_na, gb_na, rows, in_dim, H)
        torch.cuda.synchronize()
        assert rc == 0, lib.su_noalloc_strerror(rc)
        status = (ctypes.c_int * 4)()
        assert lib.su_noalloc_status(status) == 0 and status[0] == 0
        torch.testing.assert_close(dxh[:, :in_dim], dx_ref, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(dxh[:, in_dim:], dhp_ref, rtol=1e-4, atol=1e-5)
        torch.testing.assert_close(dcp, dcp_ref, rtol=1e-4, atol=1e-5)
        for a, r in zip(gw_na + gb_na, gw_ref + gb_ref):
            torch.testing.assert_close(a, r, rtol=1e-4, atol=1e-4)


def test_noalloc_rejects_oversize_and_bad_arguments():
    C, lib = _lib()
    cap = lib.su_noalloc_scratch_capacity()
    H, in_dim = 32, 64
    rows = cap // (4 * 4 * H) + 64  # gate gradients alone exceed the static array
    assert lib.su_noalloc_scratch_required(rows, in_dim, H) > cap
    x, h, c, w, b, dh, dc = _case(8, in_dim, H, 3)
    gw = [torch.zeros(H, in_dim + H, device="cuda") for _ in range(4)]
    gb = [torch.zeros(H, device="cuda") for _ in range(4)]
    # both checks run before anything is launched
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.su_lstm_cell_backward_noalloc(
        _ptr(x), None, None, _ptr(dh), _ptr(dh), None, None, *[_ptr(t) for t in w],
        _ptr(gw[0]), _ptr(gb[0]), _ptr(gw[1]), _ptr(gb[1]), _ptr(gw[2]), _ptr(gb[2]), _ptr(gw[3]), _ptr(gb[3]),
        _ptr(dh), _ptr(dh), rows, in_dim, H, stream)
    assert rc == -2 and b"scratch" in lib.su_noalloc_strerror(rc)
    rc = lib.su_lstm_cell_backward_noalloc(
        None, None, None, _ptr(dh), _ptr(dh), None, None, *[_ptr(t) for t in w],
        _ptr(gw[0]), _ptr(gb[0]), _ptr(gw[1]), _ptr(gb[1]), _ptr(gw[2]), _ptr(gb[2]), _ptr(gw[3]), _ptr(gb[3]),
        _ptr(dh), _ptr(dh), 8, in_dim, H, stream)
    assert rc == -1
    torch.cuda.synchronize()
