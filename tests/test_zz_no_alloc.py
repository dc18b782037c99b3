"""GPU test of b2m_matmul_nbits_noalloc, the allocation-free MatMulNBits entry point.

Some callers cannot allocate device memory while they run an operator: a host
application that has handed all device memory to its own pool, or an inference
loop that must not risk an out-of-memory failure or the device-wide
synchronisation cudaMalloc / cudaFree can cause. For them the library offers
one entry point whose only working memory is a fixed file-scope device array.
This test calls it through the C ABI twice in a row, with different inputs,
and checks each result against the existing entry point (b2m_matmul_nbits_dev,
FAST mode) within the fast-mode tolerance the other tests use. It also checks
that a request larger than the fixed scratch is refused with a clear error.
It lives in its own file, named to be collected last, and passes alone in a
fresh process as well as after the other tests.
"""
import ctypes

import numpy as np
import pytest

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


def test_noalloc_matches_existing_entry_point_twice():
    import torch

    rng = np.random.default_rng(2024)
    k, n = 1024, 768
    ctx = b2m.Context(0)
    w = ops.prepack_nbits(ctx, *_weights(rng, k, n), k=k, n=n, bits=4, blockSize=32)
    bias = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()
    stream = torch.cuda.current_stream().cuda_stream
    ctx.set_stream(stream)
    for call, m in enumerate((96, 200)):
        a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
        y_ref = torch.empty((m, n), device="cuda")
        y_new = torch.full((m, n), float("nan"), device="cuda")
        N.check(ctx.lib.b2m_matmul_nbits_dev(ctx.handle, ctypes.c_void_p(a.data_ptr()), m, w.handle,
                                             ctypes.c_void_p(bias.data_ptr()), N.MODE_FAST,
                                             ctypes.c_void_p(y_ref.data_ptr())))
        torch.cuda.synchronize()
        N.check(ctx.lib.b2m_matmul_nbits_noalloc(w.handle, ctypes.c_void_p(a.data_ptr()), m,
                                                 ctypes.c_void_p(bias.data_ptr()), ctypes.c_void_p(y_new.data_ptr()),
                                                 ctypes.c_void_p(stream)))
        torch.cuda.synchronize()
        assert_fast_close(y_new.cpu().numpy(), y_ref.cpu().numpy(), f"no-alloc call {call + 1} (m={m})")
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
