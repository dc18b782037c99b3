"""DynamicQuantizeLinear on the device (b2m_dynamic_quantize_linear_dev)
against the CPU restatement of opDynamicQuantizeLinear
(lib/src/onnx_ops.dart:3556-3583) and the reference fixture: bit-exact y,
scale and zero point; then the dynamic-quant chain into MatMulInteger with the
zero point read from device memory."""
import numpy as np
import pytest

import oracle
from tests.conftest import load_golden

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import onnx_runtime_dart_b200 as b2m  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = b2m.Context(0)
    yield c
    c.synchronize()


def _check(ctx, x):
    y, s, z = b2m.opDynamicQuantizeLinear(x, ctx=ctx)
    wy, ws, wz = oracle.dynamic_quantize_linear(x)
    assert s.numpy().reshape(()) == ws
    assert int(z.numpy().reshape(())) == wz
    np.testing.assert_array_equal(y.numpy(), wy)


def test_fixture(ctx):
    g = load_golden("dynamicquantizelinear")
    y, s, z = b2m.opDynamicQuantizeLinear(g["arrays"][0], ctx=ctx)
    exp = g["expected_arrays"]
    assert y.numpy().astype(np.int64).tolist() == exp["out0"].tolist()
    assert s.numpy().reshape(()) == np.float32(exp["out1"])
    assert int(z.numpy().reshape(())) == int(exp["out2"])


@pytest.mark.parametrize("n", [1, 7, 1000, 4099, (1 << 20) + 3, 8 << 20])
@pytest.mark.parametrize("dist", ["normal", "positive", "negative", "wide"])
def test_random_bit_exact(ctx, n, dist):
    rng = np.random.default_rng(n + len(dist))
    if dist == "normal":
        x = rng.standard_normal(n).astype(np.float32) * 3
    elif dist == "positive":
        x = rng.uniform(0.5, 9.0, n).astype(np.float32)
    elif dist == "negative":
        x = -rng.uniform(1e-3, 4.0, n).astype(np.float32)
    else:
        x = (rng.standard_normal(n) * np.exp(rng.uniform(-20, 20, n))).astype(np.float32)
    _check(ctx, x)


def test_zeros_and_repeat_calls(ctx):
    _check(ctx, np.zeros(1000, np.float32))
    # The block counter resets itself: back-to-back calls stay exact.
    for i in range(3):
        _check(ctx, np.random.default_rng(i).standard_normal((64, 1024)).astype(np.float32))


def test_dynamic_quant_chain_into_matmul_integer(ctx):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((64, 1024)).astype(np.float32)
    w = rng.integers(-127, 128, (1024, 3072)).astype(np.int8)
    bz = rng.integers(-4, 5, 3072).astype(np.int8)
    y, s, z = b2m.opDynamicQuantizeLinear(x, ctx=ctx)
    got = b2m.opMatMulInteger(y, ctx.prepack_i8(w), z, bz, ctx=ctx).numpy()
    wy, ws, wz = oracle.dynamic_quantize_linear(x)
    want = oracle.matmul_integer(wy, w, np.array(wz, np.uint8), bz, nthreads=8)
    np.testing.assert_array_equal(got.astype(np.int64), want)
