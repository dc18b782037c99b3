"""GPU test of b2m_matmul_nbits_noalloc, the allocation-free MatMulNBits entry point.

Some callers cannot allocate device memory while they run an operator: a host
application that has handed all device memory to its own pool, or an inference
loop that must not risk an out-of-memory failure or the device-wide
synchronisation cudaMalloc / cudaFree can cause. For them the library offers
one entry point whose only working memory is a fixed file-scope device array.

The test calls it through the C ABI twice in a row, with different inputs,
and checks each result bit for bit against the existing entry point
(b2m_matmul_nbits_dev, FAST mode), which runs the same tensor-core kernels on
the same inputs, and against the oracle's restatement of opMatMulNBits within
the fast-mode tolerance the other tests use. It also covers a call whose
activations fill the fixed array exactly, a call of four rows (which the
existing entry point serves with its GEMV instead, so only the oracle
comparison applies), and the refusal of a request one row too large. It
lives in its own file, named to be collected last, and passes alone in a
fresh process as well as after the other tests.
"""
import ctypes

import numpy as np
import pytest

import oracle
from tests.conftest import assert_fast_close

pytestmark = pytest.mark.gpu

b2m = pytest.importorskip("onnx_runtime_dart_b200")
from onnx_runtime_dart_b200 import _native as N  # noqa: E402
from onnx_runtime_dart_b200 import ops  # noqa: E402


def _weights(rng, k, n, block=32):
    nb = (k + block - 1) // block
    bq = rng.integers(0, 256, (n, nb, block // 2), dtype=np.uint8)
    sc = (np.abs(rng.normal(0, 0.02, (n, nb))) + 1e-3).astype(np.float32)
    zp = rng.integers(0, 256, (n, (nb + 1) // 2), dtype=np.uint8)
    return bq, sc, zp


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _run_both(ctx, w, a, bias, m, n, stream, with_dev=True):
    """(no-alloc result, existing entry point's result or None), as numpy."""
    import torch

    y_new = torch.full((m, n), float("nan"), device="cuda")
    y_ref = None
    if with_dev:
        y_ref = torch.full((m, n), float("nan"), device="cuda")
        N.check(ctx.lib.b2m_matmul_nbits_dev(ctx.handle, _p(a), m, w.handle, _p(bias), N.MODE_FAST, _p(y_ref)))
        torch.cuda.synchronize()
    N.check(ctx.lib.b2m_matmul_nbits_noalloc(w.handle, _p(a), m, _p(bias), _p(y_new), ctypes.c_void_p(stream)))
    torch.cuda.synchronize()
    return y_new.cpu().numpy(), None if y_ref is None else y_ref.cpu().numpy()


def test_noalloc_matches_existing_entry_point_twice():
    import torch

    rng = np.random.default_rng(2024)
    k, n = 1024, 768
    ctx = b2m.Context(0)
    bq, sc, zp = _weights(rng, k, n)
    w = ops.prepack_nbits(ctx, bq, sc, zp, k=k, n=n, bits=4, blockSize=32)
    bias_h = rng.standard_normal(n).astype(np.float32)
    bias = torch.from_numpy(bias_h).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    ctx.set_stream(stream)
    for call, m in enumerate((96, 200)):
        a_h = rng.standard_normal((m, k)).astype(np.float32)
        a = torch.from_numpy(a_h).cuda()
        got, ref = _run_both(ctx, w, a, bias, m, n, stream)
        np.testing.assert_array_equal(got, ref, err_msg=f"no-alloc call {call + 1} (m={m}) vs b2m_matmul_nbits_dev")
        want = oracle.matmul_nbits(a_h, bq, sc, zp, k, n, 32, bias=bias_h, nthreads=8)
        assert_fast_close(got, want, f"no-alloc call {call + 1} (m={m}) vs the oracle")
    ctx.set_stream(None)
    w.free()
    ctx.close()


def test_noalloc_fills_its_scratch_exactly_and_serves_few_rows():
    """M x roundup(K, 8) x 2 bytes equal to the fixed array (K = 4096,
    M = 1024): accepted, bitwise equal to the existing entry point and within
    tolerance of the oracle (so nothing spilled into the error word that
    follows the array). Then four rows, within tolerance of the oracle."""
    import torch

    rng = np.random.default_rng(99)
    k, n = 4096, 256
    m = N.NOALLOC_SCRATCH_BYTES // (k * 2)
    assert m * k * 2 == N.NOALLOC_SCRATCH_BYTES
    ctx = b2m.Context(0)
    bq, sc, zp = _weights(rng, k, n)
    w = ops.prepack_nbits(ctx, bq, sc, zp, k=k, n=n, bits=4, blockSize=32)
    bias_h = rng.standard_normal(n).astype(np.float32)
    bias = torch.from_numpy(bias_h).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    ctx.set_stream(stream)
    a_h = rng.standard_normal((m, k)).astype(np.float32)
    got, ref = _run_both(ctx, w, torch.from_numpy(a_h).cuda(), bias, m, n, stream)
    np.testing.assert_array_equal(got, ref, err_msg="no-alloc at the full scratch size vs b2m_matmul_nbits_dev")
    want = oracle.matmul_nbits(a_h, bq, sc, zp, k, n, 32, bias=bias_h, nthreads=8)
    assert_fast_close(got, want, "no-alloc at the full scratch size vs the oracle")
    a4 = rng.standard_normal((4, k)).astype(np.float32)
    got4, _ = _run_both(ctx, w, torch.from_numpy(a4).cuda(), bias, 4, n, stream, with_dev=False)
    assert_fast_close(got4, oracle.matmul_nbits(a4, bq, sc, zp, k, n, 32, bias=bias_h), "no-alloc with four rows")
    ctx.set_stream(None)
    w.free()
    ctx.close()


def test_noalloc_rejects_sizes_beyond_its_scratch():
    rng = np.random.default_rng(7)
    k, n = 4096, 64
    ctx = b2m.Context(0)
    w = ops.prepack_nbits(ctx, *_weights(rng, k, n), k=k, n=n, bits=4, blockSize=32)
    m = N.NOALLOC_SCRATCH_BYTES // (k * 2) + 1  # one row more than fits
    st = ctx.lib.b2m_matmul_nbits_noalloc(w.handle, ctypes.c_void_p(16), m, None, ctypes.c_void_p(16), None)
    assert st == N.B2M_ERR_INVALID_ARGUMENT
    assert b"exceed the fixed" in ctx.lib.b2m_last_error()
    w.free()
    ctx.close()
