"""GPU tests of the host-buffer MatMulNBits call and of the context's error
word.

b2m_matmul_nbits_host is what a caller without device tensors binds (the
reference's opMatMulNBits signature over host lists, onnx_qlinear_ops.dart:115).
Where the decode GEMV serves the call and Y is pinned host memory, the kernel
stores Y straight into it; otherwise Y goes through device memory and one
copy. Both must give the bits of the device-pointer call, b2m_matmul_nbits_dev,
which runs the same kernels on the same inputs.

The error word that bounded waits and index checks set lives in mapped host
memory and is read after the call's synchronisation. A gather with an id
outside its table (the kernel checks the id, writes zeros for that row and
records the error; nothing is read out of bounds) must surface as an
ArgumentError at the next synchronisation, and the word must be clear again
for the call after it.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

b2m = pytest.importorskip("onnx_runtime_dart_b200")
torch = pytest.importorskip("torch")
from onnx_runtime_dart_b200 import _native as N  # noqa: E402


def _p(t):
    return ctypes.c_void_p(t.data_ptr() if hasattr(t, "data_ptr") else t.ctypes.data)


@pytest.fixture(scope="module")
def ctx():
    c = b2m.Context(0)
    yield c
    c.close()


def _weight(ctx, rng, k, n):
    nb = k // 32
    bq = rng.integers(0, 256, (n, nb, 16), dtype=np.uint8)
    sc = (np.abs(rng.normal(0, 0.02, (n, nb))) + 1e-3).astype(np.float32)
    zp = rng.integers(0, 256, (n, (nb + 1) // 2), dtype=np.uint8)
    return ctx.prepack_nbits(bq, sc, zp, k, n, 4, 32)


@pytest.mark.parametrize("m,mode", [(1, N.MODE_FAST), (8, N.MODE_FAST), (1, N.MODE_PRECISE), (96, N.MODE_FAST)])
def test_host_call_matches_device_call_bitwise(ctx, m, mode):
    rng = np.random.default_rng(m + 10 * mode)
    k, n = 1024, 3072
    w = _weight(ctx, rng, k, n)
    bias = rng.standard_normal(n).astype(np.float32)
    a = rng.standard_normal((m, k)).astype(np.float32)
    lib, h = ctx.lib, ctx.handle
    a_d = torch.from_numpy(a).cuda()
    b_d = torch.from_numpy(bias).cuda()
    y_d = torch.empty((m, n), device="cuda")
    torch.cuda.synchronize()  # the context's stream does not order after torch's
    N.check(lib.b2m_matmul_nbits_dev(h, _p(a_d), m, w.handle, _p(b_d), mode, _p(y_d)))
    N.check(lib.b2m_synchronize(h))
    want = y_d.cpu().numpy()
    a_pin = torch.from_numpy(a).pin_memory()
    b_pin = torch.from_numpy(bias).pin_memory()
    y_pin = torch.full((m, n), float("nan")).pin_memory()
    y_page = np.full((m, n), np.nan, np.float32)
    for _ in range(2):  # the second call reuses the scratch and the mapped Y
        N.check(lib.b2m_matmul_nbits_host(h, _p(a_pin), m, w.handle, _p(b_pin), mode, _p(y_pin)))
        np.testing.assert_array_equal(y_pin.numpy(), want)
        N.check(lib.b2m_matmul_nbits_host(h, _p(a), m, w.handle, _p(bias), mode, _p(y_page)))
        np.testing.assert_array_equal(y_page, want)
    w.free()


def test_error_word_reports_gather_index_and_clears(ctx):
    lib, h = ctx.lib, ctx.handle
    v, d = 16, 64
    table = torch.randn((v, d), device="cuda")
    y = torch.full((3, d), 7.0, device="cuda")
    ids = torch.tensor([3, v + 5, 0], dtype=torch.int64, device="cuda")
    ids_ok = torch.tensor([1, 2, 3], dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    N.check(lib.b2m_gather_rows_dev(h, _p(table), _p(ids), _p(y), 3, v, d))
    with pytest.raises(N.ArgumentError, match="outside its table"):
        N.check(lib.b2m_synchronize(h))
    got = y.cpu()
    assert torch.equal(got[0], table[3].cpu()) and torch.equal(got[2], table[0].cpu())
    assert torch.count_nonzero(got[1]) == 0
    N.check(lib.b2m_gather_rows_dev(h, _p(table), _p(ids_ok), _p(y), 3, v, d))
    N.check(lib.b2m_synchronize(h))
    assert torch.equal(y.cpu(), table[1:4].cpu())


def test_host_call_with_library_pinned_buffers(ctx):
    """A and Y staged in b2m_host_alloc buffers (what a Dart caller would
    allocate through the ABI): the same bits as the device call."""
    rng = np.random.default_rng(5)
    k, n, m = 1024, 3072, 1
    w = _weight(ctx, rng, k, n)
    lib, h = ctx.lib, ctx.handle
    a = rng.standard_normal((m, k)).astype(np.float32)
    pa, py = ctypes.c_void_p(), ctypes.c_void_p()
    N.check(lib.b2m_host_alloc(h, a.nbytes, ctypes.byref(pa)))
    N.check(lib.b2m_host_alloc(h, m * n * 4, ctypes.byref(py)))
    try:
        ctypes.memmove(pa, a.ctypes.data, a.nbytes)
        N.check(lib.b2m_matmul_nbits_host(h, pa, m, w.handle, None, N.MODE_FAST, py))
        got = np.ctypeslib.as_array(ctypes.cast(py, ctypes.POINTER(ctypes.c_float)), shape=(m, n)).copy()
        a_d = torch.from_numpy(a).cuda()
        y_d = torch.empty((m, n), device="cuda")
        torch.cuda.synchronize()
        N.check(lib.b2m_matmul_nbits_dev(h, _p(a_d), m, w.handle, None, N.MODE_FAST, _p(y_d)))
        N.check(lib.b2m_synchronize(h))
        np.testing.assert_array_equal(got, y_d.cpu().numpy())
    finally:
        N.check(lib.b2m_host_free(h, pa))
        N.check(lib.b2m_host_free(h, py))
        w.free()


@pytest.mark.parametrize("m", [1, 96])
def test_host_call_behind_queued_device_work(ctx, m):
    """A host-buffer call enqueued right behind device work still in flight on
    the same stream (a GEMV that lets the next kernel launch early) computes on
    its own A: the copy of A is ordered before the kernel that reads it."""
    rng = np.random.default_rng(77 + m)
    k, n = 1024, 3072
    w = _weight(ctx, rng, k, n)
    lib, h = ctx.lib, ctx.handle
    a_list = [rng.standard_normal((m, k)).astype(np.float32) for _ in range(2)]
    want = []
    for a in a_list:
        a_d = torch.from_numpy(a).cuda()
        y_d = torch.empty((m, n), device="cuda")
        torch.cuda.synchronize()
        N.check(lib.b2m_matmul_nbits_dev(h, _p(a_d), m, w.handle, None, N.MODE_FAST, _p(y_d)))
        N.check(lib.b2m_synchronize(h))
        want.append(y_d.cpu().numpy())
    a0_d = torch.from_numpy(a_list[0]).cuda()
    y0_d = torch.empty((m, n), device="cuda")
    a1_pin = torch.from_numpy(a_list[1]).pin_memory()
    y1_pin = torch.empty((m, n)).pin_memory()
    torch.cuda.synchronize()
    for _ in range(20):
        for _ in range(8):  # queued work that triggers its successors early
            N.check(lib.b2m_matmul_nbits_dev(h, _p(a0_d), m, w.handle, None, N.MODE_FAST, _p(y0_d)))
        N.check(lib.b2m_matmul_nbits_host(h, _p(a1_pin), m, w.handle, None, N.MODE_FAST, _p(y1_pin)))
        np.testing.assert_array_equal(y1_pin.numpy(), want[1])
    np.testing.assert_array_equal(y0_d.cpu().numpy(), want[0])
    w.free()
