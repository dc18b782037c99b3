"""GPU tests of the declared-successor L2 prefetch (b2m_weight_set_next) and
of the decode records the GEMV reads: a prefetch hint never changes a
result, freeing either weight of a link is safe, and the record path is
bitwise equal to the plain-layout path and within the contract of the
oracle's opMatMulNBits (lib/src/onnx_qlinear_ops.dart:115-228)."""
import ctypes

import numpy as np
import pytest

import oracle
from tests.conftest import assert_fast_close

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import onnx_runtime_dart_b200 as b2m  # noqa: E402
from onnx_runtime_dart_b200 import _native as N  # noqa: E402


def _weights(rng, k, n, block=32, zp=True):
    nb = (k + block - 1) // block
    bq = rng.integers(0, 256, (n, nb, block // 2), dtype=np.uint8)
    sc = (np.abs(rng.normal(0, 0.02, (n, nb))) + 1e-3).astype(np.float32)
    z = rng.integers(0, 256, (n, (nb + 1) // 2), dtype=np.uint8) if zp else None
    return bq, sc, z


def _run(ctx, w, a, m, n, mode):
    y = torch.full((m, n), float("nan"), device="cuda")
    N.check(ctx.lib.b2m_matmul_nbits_dev(ctx.handle, ctypes.c_void_p(a.data_ptr()), m, w.handle, None, mode,
                                         ctypes.c_void_p(y.data_ptr())))
    torch.cuda.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("m,k,n,block,zp", [(1, 1024, 3072, 32, True), (8, 2048, 1024, 64, True),
                                             (3, 1000, 200, 32, False), (40, 1024, 4096, 32, True),
                                             (96, 3072, 1024, 128, True)])
def test_prefetch_hint_keeps_results_and_links_survive_free(m, k, n, block, zp):
    rng = np.random.default_rng(m + k + n)
    ctx = b2m.Context(0)
    host = [_weights(rng, k, n, block, zp) for _ in range(3)]
    ws = [ctx.prepack_nbits(bq, sc, z, k, n, 4, block) for bq, sc, z in host]
    a_h = rng.standard_normal((m, k)).astype(np.float32)
    a = torch.from_numpy(a_h).cuda()
    for mode in (N.MODE_FAST, N.MODE_PRECISE):
        plain = [_run(ctx, w, a, m, n, mode) for w in ws]
        ws[0].set_next(ws[1])
        ws[1].set_next(ws[2])
        ws[2].set_next(ws[0])
        linked = [_run(ctx, w, a, m, n, mode) for w in ws]
        for p, q in zip(plain, linked):
            np.testing.assert_array_equal(p, q)
        for (bq, sc, z), y in zip(host, linked):
            want = oracle.matmul_nbits(a_h, bq, sc, z, k, n, block, nthreads=8)
            assert_fast_close(y, want, f"m={m} k={k} n={n} block={block} mode={mode}",
                              max_rel=1e-3 if mode == N.MODE_FAST else 1e-4)
        for w in ws:
            w.set_next(None)
    # Freeing the successor drops the link; the predecessor keeps working.
    ws[0].set_next(ws[1])
    ws[1].free()
    y0 = _run(ctx, ws[0], a, m, n, N.MODE_FAST)
    np.testing.assert_array_equal(y0, _run(ctx, ws[0], a, m, n, N.MODE_FAST))
    with pytest.raises(N.ArgumentError):
        other = b2m.Context(0)
        try:
            w2 = other.prepack_nbits(*host[2], k, n, 4, block)
            ws[0].set_next(w2)
        finally:
            w2.free()
            other.close()
    for w in (ws[0], ws[2]):
        w.free()
    ctx.close()

