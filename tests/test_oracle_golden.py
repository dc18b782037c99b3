"""Pins the CPU oracle (oracle/b2m_oracle.c) to the reference's golden vectors.

The vectors are the reference's ORT-generated fixtures (tests/golden/*.json,
made by tests/golden/make_golden.py from test/fixtures/*) and its hand-computed
known answers (test/gemm_prepack_test.dart:15-55,
test/compact_tensor_test.dart:90-99, test/onnx_runtime_dart_test.dart:48-70).
Tolerances are the reference test's own. CPU only.
"""
import numpy as np
import pytest

import oracle
from oracle import glue
from tests.conftest import assert_fixture_close, golden_cases, load_golden
from tests.glue_fixtures import GLUE_CASES, run_case


def run_oracle(g):
    op, x, at = g["op_type"], g["arrays"], g["attrs"]
    if op == "MatMul":
        return oracle.matmul(x[0], x[1])
    if op == "Gemm":
        return oracle.gemm(x[0], x[1], x[2] if len(x) > 2 else None, alpha=at.get("alpha", 1.0),
                           beta=at.get("beta", 1.0), transA=bool(at.get("transA", 0)),
                           transB=bool(at.get("transB", 0)))
    if op == "MatMulInteger":
        return oracle.matmul_integer(x[0], x[1], x[2] if len(x) > 2 else None, x[3] if len(x) > 3 else None)
    if op == "QLinearMatMul":
        # lo/hi from the y_zero_point's element type (onnx_graph.dart:2903, 2913-2914)
        int8 = g["inputs"][7]["tensor"]["elem_type"] == 3
        return oracle.qlinear_matmul(x[0], x[1], x[2], x[3], x[4], x[5], x[6], x[7],
                                     -128 if int8 else 0, 127 if int8 else 255)
    if op == "MatMulNBits":
        return oracle.matmul_nbits(x[0], x[1], x[2], x[3] if len(x) > 3 else None, at["K"], at["N"],
                                   at["block_size"], bias=x[5] if len(x) > 5 else None)
    if op == "Conv":
        return oracle.conv_f32(x[0], x[1], x[2] if len(x) > 2 else None, at.get("strides"), at.get("pads"),
                               at.get("dilations"), at.get("group", 1), at.get("auto_pad", "NOTSET"))
    if op == "ConvInteger":
        return oracle.conv_integer(x[0], x[1], x[2] if len(x) > 2 else None, x[3] if len(x) > 3 else None,
                                   at.get("strides"), at.get("pads"), at.get("dilations"), at.get("group", 1))
    if op == "QLinearConv":
        int8 = g["inputs"][7]["tensor"]["elem_type"] == 3
        return oracle.qlinear_conv(x[0], x[1], x[2], x[3], x[4], x[5], x[6], x[7], x[8] if len(x) > 8 else None,
                                   at.get("strides"), at.get("pads"), at.get("dilations"), at.get("group", 1),
                                   -128 if int8 else 0, 127 if int8 else 255)
    if op == "ConvTranspose":
        return oracle.conv_transpose_f32(x[0], x[1], x[2] if len(x) > 2 else None, at.get("strides"), at.get("pads"),
                                         at.get("dilations"), at.get("output_padding"), at.get("output_shape"),
                                         at.get("group", 1))
    pytest.skip(f"{op} is not a MatMul-family op")


@pytest.mark.parametrize("case", [c for c in golden_cases() if not c.startswith("dynamic") and c not in GLUE_CASES])
def test_oracle_matches_reference_fixture(case):
    g = load_golden(case)
    got = run_oracle(g)
    assert_fixture_close(got, g["expected_arrays"][g["outputs"][0]], case)


def test_gemm_prepack_known_answer():
    # test/gemm_prepack_test.dart:15-55: X[2x3] . W[4x3]^T + C[4]
    w = np.arange(1, 13, dtype=np.float32).reshape(4, 3)
    c = np.array([10, 20, 30, 40], np.float32)
    x = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    y = oracle.gemm(x, w, c, transB=True)
    assert y.ravel().tolist() == [24.0, 52.0, 80.0, 108.0, 42.0, 97.0, 152.0, 207.0]


def test_matmul_integer_compact_known_answer():
    # test/compact_tensor_test.dart:90-99
    a = np.array([[10, 130, 250]], np.uint8)
    b = np.array([-1, 2, 3, -4, 5, 6], np.int8).reshape(3, 2)
    assert oracle.matmul_integer(a, b, np.array(10), np.array(1)).ravel().tolist() == [1200, 600]


def test_matmul_identity_known_answer():
    # test/onnx_runtime_dart_test.dart:48-70
    x = np.array([[5, 6], [7, 8]], np.float32)
    assert oracle.matmul(x, np.eye(2, dtype=np.float32)).ravel().tolist() == [5, 6, 7, 8]


@pytest.mark.parametrize("m", range(1, 7))
def test_matmul_kernel_small_shapes_vs_double(m):
    # test/gemm_kernel_test.dart:45-60: every m,k,n in 1..6 within 1e-5 of a
    # double-accumulating naive loop.
    rng = np.random.default_rng(11)
    for k in range(1, 7):
        for n in range(1, 7):
            a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
            b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
            got = oracle.matmul_kernel(a, b, m, k, n)
            want = (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)
            np.testing.assert_allclose(got, want, atol=1e-5, rtol=0)


@pytest.mark.parametrize("mkn", [(1, 384, 384), (33, 65, 17), (7, 128, 5), (128, 64, 128), (5, 1, 9),
                                 (64, 384, 1), (1, 40, 151), (1, 128, 19), (1, 896, 512)])
def test_matmul_kernel_odd_shapes(mkn):
    # test/gemm_kernel_test.dart:62-80
    m, k, n = mkn
    rng = np.random.default_rng(sum(mkn))
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    got = oracle.matmul_kernel(a, b, m, k, n)
    want = a.astype(np.float64) @ b.astype(np.float64)
    assert np.max(np.abs(got - want)) < 1e-4


def test_float_lane_vs_double_tail_rules():
    # m < 4 tail columns (n % 4) accumulate in double, everything else in
    # float32 lanes (gemm_kernel_simd.dart:601-608, 665-672).
    rng = np.random.default_rng(5)
    m, k, n = 2, 257, 7
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    got = oracle.matmul_kernel(a, b, m, k, n)
    f32 = np.zeros((m, n), np.float32)
    for kk in range(k):
        f32 = (f32 + (a[:, kk:kk + 1] * b[kk:kk + 1, :]).astype(np.float32)).astype(np.float32)
    dbl = (a.astype(np.float64) @ b.astype(np.float64)).astype(np.float32)
    np.testing.assert_array_equal(got[:, :4], f32[:, :4])
    np.testing.assert_array_equal(got[:, 4:], dbl[:, 4:])


def test_threads_are_bitwise_neutral():
    # The pool's contract (parallel_pool.dart:7-8): column splits are bitwise identical.
    rng = np.random.default_rng(3)
    a = rng.standard_normal((9, 300)).astype(np.float32)
    b = rng.standard_normal((300, 77)).astype(np.float32)
    np.testing.assert_array_equal(oracle.matmul(a, b, nthreads=1), oracle.matmul(a, b, nthreads=5))
    q = rng.integers(0, 256, (77, 10, 16), dtype=np.uint8)
    s = np.abs(rng.standard_normal((77, 10))).astype(np.float32)
    x = rng.standard_normal((5, 300)).astype(np.float32)
    r1 = oracle.matmul_nbits(x, q, s, None, 300, 77, 32, nthreads=1)
    r5 = oracle.matmul_nbits(x, q, s, None, 300, 77, 32, nthreads=5)
    np.testing.assert_array_equal(r1, r5)


def test_round_even_and_multiplier():
    # _roundEven (onnx_qlinear_ops.dart:19-26)
    assert [oracle.round_even(v) for v in (0.5, 1.5, 2.5, -0.5, -1.5, 2.4999, -2.6)] == [0, 2, 2, 0, -2, 2, -3]
    m = oracle.qlinear_multiplier(0.02, 0.05, 0.1)
    assert m == np.float32(np.float32(np.float32(0.02) * np.float32(0.05)) / np.float32(0.1))


def test_dynamic_quantize_linear_fixture():
    # test/fixtures/dynamicquantizelinear: [y, scale, zero point] bit-exact.
    g = load_golden("dynamicquantizelinear")
    y, scale, zp = oracle.dynamic_quantize_linear(g["arrays"][0])
    exp = g["expected_arrays"]
    assert y.astype(np.int64).tolist() == exp["out0"].tolist()
    assert np.float32(scale) == np.float32(exp["out1"])
    assert zp == int(exp["out2"])


def test_dynamic_quantize_linear_edges():
    # Range always spans 0; all-zero input gives scale 0, zp 0, y 0.
    y, s, z = oracle.dynamic_quantize_linear(np.zeros(5, np.float32))
    assert s == 0 and z == 0 and y.tolist() == [0] * 5
    y, s, z = oracle.dynamic_quantize_linear(np.array([1.0, 2.0, 255.0], np.float32))
    assert z == 0 and s == np.float32(1.0) and y.tolist() == [1, 2, 255]
    y, s, z = oracle.dynamic_quantize_linear(np.array([-255.0, -1.0], np.float32))
    assert z == 255 and y.tolist() == [0, 254]
    # ties go to even: 0.5 / 1 and 2.5 / 1 with scale 1
    y, s, z = oracle.dynamic_quantize_linear(np.array([0.5, 2.5, 255.0], np.float32))
    assert y.tolist() == [0, 2, 255]


class _OracleGlue:
    """oracle/glue.py behind the fixture runner's interface."""

    @staticmethod
    def gelu(x):
        return glue.gelu(x)

    @staticmethod
    def rmsnorm(x, gamma, eps, skip):
        return glue.rmsnorm(x, gamma, eps, skip=skip)

    @staticmethod
    def argmax_last(x):
        return glue.argmax(x)

    @staticmethod
    def rotary(x, pos, cos, sin, heads, interleaved):
        return glue.rotary(x, np.asarray(pos), cos, sin, heads, interleaved)

    @staticmethod
    def gqa(q, k, v, h, kvh, pk, pv, cos, sin, scale):
        return glue.gqa(q, k, v, h, kvh, pk, pv, cos, sin, scale=scale or None)

    @staticmethod
    def mha(q, k, v, h, bias, scale):
        return glue.mha(q, k, v, h, h, bias4d=bias, scale=scale or None)


@pytest.mark.parametrize("case", GLUE_CASES)
def test_glue_oracle_matches_reference_fixture(case):
    g = load_golden(case)
    got = run_case(g, _OracleGlue)
    for name, arr in got.items():
        want = g["expected_arrays"][name]
        if want.dtype.kind in "iu":
            assert np.asarray(arr).astype(np.int64).tolist() == want.tolist(), f"{case}:{name}"
        else:
            assert_fixture_close(arr, want, f"{case}:{name}")


def _conv_naive_double(x, w, bias, s, p, d, group):
    """Direct 2-D convolution in float64 (test-only cross-check)."""
    n, cin, h, wd = x.shape
    m, cpg, kh, kw = w.shape
    oh = (h + p[0] + p[2] - (d[0] * (kh - 1) + 1)) // s[0] + 1
    ow = (wd + p[1] + p[3] - (d[1] * (kw - 1) + 1)) // s[1] + 1
    xp = np.zeros((n, cin, h + p[0] + p[2], wd + p[1] + p[3]))
    xp[:, :, p[0]:p[0] + h, p[1]:p[1] + wd] = x
    out = np.zeros((n, m, oh, ow))
    mpg = m // group
    for om in range(m):
        g = om // mpg
        for ky in range(kh):
            for kx in range(kw):
                patch = xp[:, g * cpg:(g + 1) * cpg, ky * d[0]:ky * d[0] + s[0] * (oh - 1) + 1:s[0],
                           kx * d[1]:kx * d[1] + s[1] * (ow - 1) + 1:s[1]]
                out[:, om] += np.einsum("nchw,c->nhw", patch, w[om, :, ky, kx].astype(np.float64))
        if bias is not None:
            out[:, om] += bias[om]
    return out


@pytest.mark.parametrize("cfg", [
    # (n, cin, h, w, m, kh, kw, stride, pad, dil, group)
    (2, 3, 9, 11, 8, 3, 3, 1, 1, 1, 1),
    (1, 4, 8, 8, 2, 3, 3, 2, 0, 1, 1),      # m < 4: double tail pixels
    (1, 6, 7, 9, 6, 3, 2, 1, 1, 2, 3),      # groups, 2 outputs per group
    (2, 8, 5, 5, 16, 1, 1, 1, 0, 1, 1),     # pointwise
    (1, 4, 10, 10, 4, 5, 5, 1, 2, 1, 4),    # depthwise
])
def test_conv_oracle_vs_float64(cfg):
    n, cin, h, wd, m, kh, kw, st, pd, dl, grp = cfg
    rng = np.random.default_rng(7)
    x = rng.standard_normal((n, cin, h, wd)).astype(np.float32)
    w = (rng.standard_normal((m, cin // grp, kh, kw)) / np.sqrt(cin // grp * kh * kw)).astype(np.float32)
    b = rng.standard_normal(m).astype(np.float32)
    got = oracle.conv_f32(x, w, b, [st, st], [pd] * 4, [dl, dl], grp)
    want = _conv_naive_double(x, w, b, [st, st], [pd] * 4, [dl, dl], grp)
    assert got.shape == want.shape
    assert np.max(np.abs(got - want)) <= 1e-5 * max(1.0, np.max(np.abs(want)))


def test_conv_oracle_chunking_is_per_row():
    """Chunking the im2col panel over output rows (onnx_nn_ops.dart:313-323)
    leaves every element's k order alone: with m >= 4 a conv too large for one
    chunk equals the row-by-row direct fp32 evaluation in k order."""
    rng = np.random.default_rng(3)
    x = rng.standard_normal((1, 64, 40, 1100)).astype(np.float32)   # colRows*ow = 576*1100 > (8<<20)/16
    w = (rng.standard_normal((4, 64, 3, 3)) * 0.05).astype(np.float32)
    got = oracle.conv_f32(x, w, None, [1, 1], [1, 1, 1, 1], [1, 1], 1)
    # Reference per element: float acc += float(a*b) in (c, ky, kx) order.
    xp = np.zeros((64, 42, 1102), np.float32)
    xp[:, 1:41, 1:1101] = x[0]
    oy, ox = 17, 1099
    for om in range(4):
        acc = np.float32(0)
        for c in range(64):
            for ky in range(3):
                for kx in range(3):
                    acc = np.float32(acc + np.float32(w[om, c, ky, kx] * xp[c, oy + ky, ox + kx]))
        assert got[0, om, oy, ox] == acc


def _conv_transpose_f64(x, w, bias, s, p, d, op, group):
    n, cin = x.shape[:2]
    nd = x.ndim - 2
    mpg = w.shape[1]
    ks = w.shape[2:]
    osp = [(x.shape[2 + a] - 1) * s[a] + d[a] * (ks[a] - 1) + 1 + op[a] - p[a] - p[nd + a] for a in range(nd)]
    out = np.zeros([n, mpg * group] + osp)
    cpg = cin // group
    for idx in np.ndindex(*x.shape[2:]):
        for kidx in np.ndindex(*ks):
            o = [idx[a] * s[a] + kidx[a] * d[a] - p[a] for a in range(nd)]
            if any(o[a] < 0 or o[a] >= osp[a] for a in range(nd)):
                continue
            for g in range(group):
                xs = x[(slice(None), slice(g * cpg, (g + 1) * cpg)) + idx].astype(np.float64)   # [n, cpg]
                ws = w[(slice(g * cpg, (g + 1) * cpg), slice(None)) + kidx].astype(np.float64)  # [cpg, mpg]
                out[(slice(None), slice(g * mpg, (g + 1) * mpg)) + tuple(o)] += xs @ ws
    if bias is not None:
        out += bias.reshape([1, -1] + [1] * nd)
    return out


@pytest.mark.parametrize("cfg", [
    # (n, cin, spatial, mpg, kernel, strides, pads, dilations, output_padding, group)
    (1, 4, (6, 7), 3, (3, 2), (2, 1), (1, 0, 0, 1), (1, 2), (1, 0), 2),   # GEMM + overlap-add path
    (2, 3, (5, 5), 2, (3, 3), (2, 2), (1, 1, 1, 1), (1, 1), (0, 0), 1),   # generic scatter (two images)
    (1, 2, (9,), 4, (5,), (3,), (2, 1), (1,), (2,), 1),                   # 1-D GEMM path
    (1, 2, (3, 4, 3), 2, (2, 2, 2), (1, 2, 1), (0, 0, 0, 0, 1, 0), (1, 1, 1), (0, 0, 0), 1),  # 3-D
])
def test_conv_transpose_oracle_vs_float64(cfg):
    n, cin, sp, mpg, ks, s, p, d, op, grp = cfg
    rng = np.random.default_rng(len(sp) + cin)
    x = rng.standard_normal((n, cin, *sp)).astype(np.float32)
    w = (rng.standard_normal((cin, mpg, *ks)) * 0.3).astype(np.float32)
    b = rng.standard_normal(mpg * grp).astype(np.float32)
    got = oracle.conv_transpose_f32(x, w, b, s, p, d, op, None, grp)
    want = _conv_transpose_f64(x, w, b, s, p, d, op, grp)
    assert got.shape == want.shape
    assert np.max(np.abs(got - want)) <= 1e-5 * max(1.0, np.max(np.abs(want)))


# --- opConv's Winograd F(2x2, 3x3) branch -----------------------------------

def _conv3x3_f64(x, w, b, pad):
    x, w = x.astype(np.float64), w.astype(np.float64)
    oh, ow = x.shape[2] + 2 * pad - 2, x.shape[3] + 2 * pad - 2
    xp = np.pad(x, ((0, 0), (0, 0), (pad, pad), (pad, pad)))
    out = np.zeros((x.shape[0], w.shape[0], oh, ow))
    for ky in range(3):
        for kx in range(3):
            out += np.einsum("nchw,mc->nmhw", xp[:, :, ky:ky + oh, kx:kx + ow], w[:, :, ky, kx])
    return out + (0 if b is None else b.astype(np.float64)[None, :, None, None])


@pytest.mark.parametrize("case,pad", [("conv2d_basic", 0), ("conv2d_bias", 0), ("conv2d_pads", 1)])
def test_winograd_restatement_matches_eligible_shaped_fixtures(case, pad):
    """The reference's 3x3 stride-1 group-1 fixtures with all-0 / all-1 pads
    (the branch's shapes; the executor itself takes it from 1024 output
    pixels on) through the Winograd restatement, at the fixture tolerance."""
    g = load_golden(case)
    x = g["arrays"]
    got = oracle.conv_winograd_f32(x[0], x[1], x[2] if len(x) > 2 else None, pad=pad)
    assert_fixture_close(got, g["expected_arrays"][g["outputs"][0]], case + " (Winograd)")


@pytest.mark.parametrize("n,c,h,w,m,pad", [
    (2, 16, 34, 34, 8, 1),      # one band
    (1, 3, 40, 33, 2, 0),       # two output channels: double tail columns in the products
    (1, 1024, 256, 16, 4, 1),   # two bands of tile rows (127 + 1)
    (1, 1024, 230, 18, 2, 1),   # two bands with tail columns of different widths
])
def test_winograd_restatement_against_float64(n, c, h, w, m, pad):
    """Eligible shapes, banding included, against a float64 convolution at
    the fixture tolerance; the im2col restatement (what the device EXACT
    kernels reproduce) meets the same bound, so the two branches differ by
    float32 rounding only."""
    rng = np.random.default_rng(c + h)
    x = rng.standard_normal((n, c, h, w)).astype(np.float32)
    wt = (rng.standard_normal((m, c, 3, 3)) / np.sqrt(9 * c)).astype(np.float32)
    b = rng.standard_normal(m).astype(np.float32)
    assert oracle.conv_winograd_eligible(wt.shape, x.shape, pads=[pad] * 4)
    ref = _conv3x3_f64(x, wt, b, pad)
    assert_fixture_close(oracle.conv_winograd_f32(x, wt, b, pad=pad), ref, "Winograd vs float64")
    assert_fixture_close(oracle.conv_f32(x, wt, b, pads=[pad] * 4), ref, "im2col vs float64")


def test_winograd_eligibility_mirrors_the_reference():
    """convWinogradEligible (lib/src/onnx_nn_ops.dart:779-812)."""
    e = oracle.conv_winograd_eligible
    assert e((8, 4, 3, 3), (1, 4, 32, 32), pads=[1, 1, 1, 1])          # 32 x 32 = 1024 outputs
    assert not e((8, 4, 3, 3), (1, 4, 31, 32), pads=[1, 1, 1, 1])      # 992
    assert e((8, 4, 3, 3), (1, 4, 34, 34), pads=[0, 0, 0, 0])
    assert not e((8, 4, 3, 3), (1, 4, 64, 64), pads=[1, 0, 1, 0])      # mixed pads
    assert not e((8, 4, 3, 3), (1, 4, 64, 64), pads=None)              # pads must be given
    assert not e((8, 4, 3, 3), (1, 4, 64, 64), pads=[1] * 4, strides=[2, 2])
    assert not e((8, 4, 3, 3), (1, 4, 64, 64), pads=[1] * 4, dilations=[2, 2])
    assert not e((8, 2, 3, 3), (1, 4, 64, 64), pads=[1] * 4, group=2)
    assert not e((8, 4, 5, 5), (1, 4, 64, 64), pads=[1] * 4)
    assert not e((8, 4, 3, 3), (1, 4, 64, 64), pads=[1] * 4, auto_pad="SAME_UPPER")
