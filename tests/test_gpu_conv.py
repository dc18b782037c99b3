"""GPU parity of the convolutions that run through the GEMM cores (Conv,
ConvInteger, QLinearConv), through the C ABI, against the CPU oracle.

Bars (written here, per op):
  * Conv, mode EXACT: bitwise equal to the oracle's restatement of opConv's
    im2col / depthwise / N-D arithmetic (lib/src/onnx_nn_ops.dart:179-545).
  * Conv, mode FAST (bf16 split planes on tcgen05): max|d|/max|ref| <= 1e-3
    and cosine >= 0.99999 against the oracle (the path's float contract).
  * ConvInteger / QLinearConv: bitwise equal (integers).
The reference's own fixtures run through the dispatch hook in
test_gpu_parity.py (test_golden_fixture_via_dispatch).
"""
import numpy as np
import pytest

import oracle
from tests.conftest import assert_fast_close

pytestmark = pytest.mark.gpu

b2m = pytest.importorskip("onnx_runtime_dart_b200")
from onnx_runtime_dart_b200 import _native as N  # noqa: E402
from onnx_runtime_dart_b200 import ops  # noqa: E402
from onnx_runtime_dart_b200.dispatch import GpuDispatch  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = b2m.Context(0)
    yield c
    c.synchronize()


def _conv_case(rng, n, cin, sp, m, ks, group, bias=True):
    x = rng.standard_normal((n, cin, *sp)).astype(np.float32)
    fan = cin // group * int(np.prod(ks))
    w = (rng.standard_normal((m, cin // group, *ks)) / np.sqrt(fan)).astype(np.float32)
    b = rng.standard_normal(m).astype(np.float32) if bias else None
    return x, w, b


# (n, cin, spatial, m, kernel, strides, pads, dilations, group, auto_pad)
F32_CASES = [
    (2, 3, (9, 11), 8, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, "NOTSET"),
    (1, 4, (8, 8), 2, (3, 3), (2, 2), (0, 0, 0, 0), (1, 1), 1, "NOTSET"),       # 2 outputs: double tails
    (1, 6, (7, 9), 6, (3, 2), (1, 1), (1, 0, 2, 1), (2, 1), 3, "NOTSET"),       # groups, asymmetric pads
    (2, 8, (5, 5), 16, (1, 1), (1, 1), (0, 0, 0, 0), (1, 1), 1, "NOTSET"),      # pointwise
    (1, 4, (10, 10), 4, (5, 5), (1, 1), (2, 2, 2, 2), (1, 1), 4, "NOTSET"),     # depthwise
    (1, 3, (7, 7), 5, (3, 3), (2, 2), None, (1, 1), 1, "SAME_UPPER"),
    (1, 3, (7, 8), 5, (3, 3), (2, 3), None, (1, 1), 1, "SAME_LOWER"),
    (1, 3, (9, 9), 5, (3, 3), (2, 2), None, (1, 1), 1, "VALID"),
    (3, 5, (17,), 7, (4,), (2,), (1, 2), (2,), 1, "NOTSET"),                    # 1-D
    (2, 4, (19,), 4, (3,), (1,), (1, 1), (1,), 4, "NOTSET"),                    # 1-D depthwise
    (1, 2, (5, 6, 7), 3, (3, 3, 2), (1, 2, 1), (1, 1, 0, 1, 0, 1), (1, 1, 2), 1, "NOTSET"),  # 3-D
    (4, 64, (28, 28), 96, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, "NOTSET"),   # a ResNet-style layer
    (2, 32, (14, 14), 64, (3, 3), (2, 2), (1, 1, 1, 1), (1, 1), 2, "NOTSET"),   # grouped, strided
]


@pytest.mark.parametrize("case", F32_CASES, ids=[f"cfg{i}" for i in range(len(F32_CASES))])
def test_conv_f32_exact_and_fast(ctx, case):
    n, cin, sp, m, ks, st, pd, dl, grp, ap = case
    rng = np.random.default_rng(len(sp) * 100 + m)
    x, w, b = _conv_case(rng, n, cin, sp, m, ks, grp)
    want = oracle.conv_f32(x, w, b, st, pd, dl, grp, ap)
    pw = ctx.prepack_conv(w)
    kw = dict(strides=st, pads=pd, dilations=dl, group=grp, autoPad=ap, ctx=ctx)
    exact = ops.opConv(x, pw, b, mode=ops.MODE_EXACT, **kw).numpy()
    assert exact.shape == want.shape
    np.testing.assert_array_equal(exact, want)
    fast = ops.opConv(x, pw, b, mode=ops.MODE_FAST, **kw).numpy()
    assert_fast_close(fast, want, f"conv fast {case}")


def test_conv_f32_exact_chunked_double_tails(ctx):
    """Two outputs per group and an im2col panel of several row chunks: the
    last n % 4 pixels of every chunk accumulate in double, as matmulKernel's
    small-m paths do (gemm_kernel_simd.dart:601-608, 665-672)."""
    rng = np.random.default_rng(11)
    x, w, b = _conv_case(rng, 1, 64, (40, 1100), 2, (3, 3), 1)
    want = oracle.conv_f32(x, w, b, (1, 1), (1, 1, 1, 1), (1, 1), 1)
    got = ops.opConv(x, ctx.prepack_conv(w), b, pads=(1, 1, 1, 1), mode=ops.MODE_EXACT, ctx=ctx).numpy()
    np.testing.assert_array_equal(got, want)


def test_conv_device_chain_and_errors(ctx):
    rng = np.random.default_rng(5)
    x, w, b = _conv_case(rng, 2, 4, (6, 6), 8, (3, 3), 1)
    pw = ctx.prepack_conv(w)
    y1 = ops.opConv(x, pw, b, pads=(1, 1, 1, 1), ctx=ctx)            # stays on the device
    w2 = (rng.standard_normal((4, 8, 1, 1)) * 0.3).astype(np.float32)
    y2 = ops.opConv(y1, ctx.prepack_conv(w2), None, ctx=ctx).numpy()
    want = oracle.conv_f32(oracle.conv_f32(x, w, b, None, (1, 1, 1, 1)), w2)
    np.testing.assert_array_equal(y2, want)
    with pytest.raises(N.ArgumentError, match="channel mismatch"):
        ops.opConv(rng.standard_normal((1, 5, 6, 6)).astype(np.float32), pw, ctx=ctx)
    with pytest.raises(N.UnsupportedError, match="1-3 spatial dims"):
        ops.opConv(rng.standard_normal((1, 4, 2, 2, 2, 2)).astype(np.float32), pw, ctx=ctx)
    with pytest.raises(N.ArgumentError, match="bias"):
        ops.opConv(x, pw, np.zeros(3, np.float32), ctx=ctx)
    d = GpuDispatch(ctx, {"w": w}, {})
    with pytest.raises(N.StateError, match="kernel_shape"):
        d.dispatch("Conv", ["x", "w"], [x, w], {"kernel_shape": [2, 2]})


def _int_case(rng, n, cin, sp, m, ks, xdt, wdt):
    lo_x, hi_x = (0, 256) if xdt == np.uint8 else (-128, 128)
    lo_w, hi_w = (0, 256) if wdt == np.uint8 else (-128, 128)
    x = rng.integers(lo_x, hi_x, (n, cin, *sp)).astype(xdt)
    w = rng.integers(lo_w, hi_w, (m, *ks)).astype(wdt)
    return x, w


# (n, cin, spatial, m, kernel, strides, pads, dilations, group, x dtype, w dtype, per-channel w_zp)
INT_CASES = [
    (1, 2, (5, 5), 3, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, np.uint8, np.int8, False),
    (2, 16, (20, 20), 64, (3, 3), (1, 1), (1, 1, 1, 1), (1, 1), 1, np.uint8, np.int8, True),   # tensor cores
    (2, 3, (33, 31), 40, (3, 3), (2, 2), (1, 1, 1, 1), (1, 1), 1, np.uint8, np.uint8, False),  # k 27 -> 32
    (1, 8, (9, 9), 12, (3, 3), (1, 1), (0, 1, 2, 0), (2, 1), 4, np.int8, np.int8, True),      # groups of 3
    (1, 4, (11, 7), 128, (2, 2), (1, 2), (1, 1, 1, 1), (1, 1), 4, np.uint8, np.int8, True),    # groups of 32
    (2, 3, (12,), 4, (5,), (1,), (2, 2), (1,), 1, np.uint8, np.int8, False),                   # 1-D
]


@pytest.mark.parametrize("case", INT_CASES, ids=[f"cfg{i}" for i in range(len(INT_CASES))])
def test_conv_integer_bit_exact(ctx, case):
    n, cin, sp, m, ks, st, pd, dl, grp, xdt, wdt, per_ch = case
    rng = np.random.default_rng(m + cin)
    x, w = _int_case(rng, n, cin, sp, m, (cin // grp, *ks), xdt, wdt)
    xz = np.array(rng.integers(0, 256) if xdt == np.uint8 else rng.integers(-128, 128), xdt)
    wz = (rng.integers(-4, 5, m) if wdt == np.int8 else rng.integers(120, 136, m)).astype(wdt)
    if not per_ch:
        wz = wz[:1].reshape(())
    want = oracle.conv_integer(x, w, xz, wz, st, pd, dl, grp)
    got = ops.opConvInteger(x, ctx.prepack_conv(w), xz, wz, strides=st, pads=pd, dilations=dl, group=grp,
                            ctx=ctx).numpy()
    assert got.dtype == np.int32
    np.testing.assert_array_equal(got.astype(np.int64), want)


@pytest.mark.parametrize("case", INT_CASES[:5], ids=[f"cfg{i}" for i in range(5)])
@pytest.mark.parametrize("out_int8", [False, True])
def test_qlinear_conv_bit_exact(ctx, case, out_int8):
    n, cin, sp, m, ks, st, pd, dl, grp, xdt, wdt, per_ch = case
    rng = np.random.default_rng(3 * m + cin)
    x, w = _int_case(rng, n, cin, sp, m, (cin // grp, *ks), xdt, wdt)
    xz = np.array(rng.integers(0, 256) if xdt == np.uint8 else rng.integers(-128, 128), xdt)
    wz = (rng.integers(-4, 5, m) if wdt == np.int8 else rng.integers(120, 136, m)).astype(wdt)
    ws = (np.abs(rng.normal(0.01, 0.004, m)) + 1e-3).astype(np.float32)
    if not per_ch:
        wz, ws = wz[:1].reshape(()), ws[:1]
    xs, ys = np.float32(0.02), np.float32(0.9 if cin * np.prod(ks) > 50 else 0.2)
    bias = rng.integers(-5000, 5000, m).astype(np.int32)
    lo, hi = (-128, 127) if out_int8 else (0, 255)
    yz = np.array(3 if out_int8 else 120, np.int8 if out_int8 else np.uint8)
    want = oracle.qlinear_conv(x, xs, xz, w, ws, wz, ys, yz, bias, st, pd, dl, grp, lo, hi)
    got = ops.opQLinearConv(x, xs, xz, ctx.prepack_conv(w), ws, wz, ys, yz, bias, strides=st, pads=pd,
                            dilations=dl, group=grp, lo=lo, hi=hi, ctx=ctx).numpy()
    assert got.dtype == (np.int8 if out_int8 else np.uint8)
    np.testing.assert_array_equal(got.astype(np.int64), want)
    assert 0 < np.count_nonzero((want > lo) & (want < hi))  # not all saturated


def test_conv_integer_errors(ctx):
    rng = np.random.default_rng(2)
    x, w = _int_case(rng, 1, 2, (5, 5), 3, (2, 3, 3), np.uint8, np.int8)
    pw = ctx.prepack_conv(w)
    with pytest.raises(N.UnsupportedError, match="scalar or per-output-channel"):
        ops.opConvInteger(x, pw, None, np.zeros(2, np.int8), ctx=ctx)
    with pytest.raises(N.UnsupportedError, match="1-D/2-D"):
        ops.opConvInteger(x.reshape(1, 2, 5, 5, 1), pw, ctx=ctx)
    with pytest.raises(N.UnsupportedError, match="2-D"):
        ops.opQLinearConv(x.reshape(1, 2, 25), 0.1, None, pw, np.float32([0.1]), None, 0.1, None, lo=0, hi=255,
                          ctx=ctx)


# (n, cin, spatial, mpg, kernel, strides, pads, dilations, output_padding, output_shape, group)
CT_CASES = [
    (1, 4, (6, 7), 3, (3, 2), (2, 1), (1, 0, 0, 1), (1, 2), (1, 0), None, 2),      # GEMM + overlap-add
    (1, 16, (14, 14), 8, (4, 4), (2, 2), (1, 1, 1, 1), (1, 1), (0, 0), None, 1),  # decoder-style upsampling
    (1, 2, (9,), 4, (5,), (3,), (2, 1), (1,), (2,), None, 1),                     # 1-D GEMM path
    (1, 2, (5,), 1, (3,), (1,), (0, 0), (1,), (0,), None, 1),                     # 3 planes: double tails
    (2, 3, (5, 5), 2, (3, 3), (2, 2), (1, 1, 1, 1), (1, 1), (0, 0), None, 1),     # two images: scatter
    (1, 2, (5, 5), 3, (3, 3), (2, 2), None, (1, 1), (0, 0), (10, 10), 1),         # output_shape: scatter
    (1, 2, (3, 4, 3), 2, (2, 2, 2), (1, 2, 1), (0, 0, 0, 0, 1, 0), (1, 1, 1), (0, 0, 0), None, 1),  # 3-D
]


@pytest.mark.parametrize("case", CT_CASES, ids=[f"cfg{i}" for i in range(len(CT_CASES))])
def test_conv_transpose_bitwise(ctx, case):
    n, cin, sp, mpg, ks, st, pd, dl, op, osh, grp = case
    rng = np.random.default_rng(cin * 10 + len(sp))
    x = rng.standard_normal((n, cin, *sp)).astype(np.float32)
    x[x > 1.5] = 0.0  # zero inputs, which the reference's scatter skips
    w = (rng.standard_normal((cin, mpg, *ks)) * 0.3).astype(np.float32)
    b = rng.standard_normal(mpg * grp).astype(np.float32)
    want = oracle.conv_transpose_f32(x, w, b, st, pd, dl, op, osh, grp)
    got = ops.opConvTranspose(x, w, b, strides=st, pads=pd, dilations=dl, outputPadding=op, outputShape=osh,
                              group=grp, ctx=ctx).numpy()
    assert got.shape == want.shape
    np.testing.assert_array_equal(got, want)


def test_conv_transpose_errors(ctx):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((1, 4, 5, 5)).astype(np.float32)
    w = rng.standard_normal((4, 2, 3, 3)).astype(np.float32)
    with pytest.raises(N.ArgumentError, match="channel mismatch"):
        ops.opConvTranspose(x, w[:3], ctx=ctx)
    with pytest.raises(N.ArgumentError, match="rank"):
        ops.opConvTranspose(x, w[:, :, :, 0], ctx=ctx)
    with pytest.raises(N.ArgumentError, match="bias"):
        ops.opConvTranspose(x, w, np.zeros(3, np.float32), ctx=ctx)
    d = GpuDispatch(ctx, {"w": w}, {})
    with pytest.raises(N.StateError, match="kernel_shape"):
        d.dispatch("ConvTranspose", ["x", "w"], [x, w], {"kernel_shape": [2, 2]})
