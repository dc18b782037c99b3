"""GPU parity: the CUDA kernels (through the C ABI) against the CPU oracle.

Bars (written here, per op):
  * fp32 MatMul / Gemm, mode EXACT: bitwise equal to the oracle's restatement
    of the reference Dart kernels.
  * MatMulInteger / QLinearMatMul: bitwise equal (integers).
  * MatMulNBits, mode EXACT: bitwise equal; mode FAST: max|d|/max|ref| <= 1e-3
    and cosine >= 0.99999 against the oracle.
  * The reference's own golden fixtures: its tolerance (max|d| <=
    max(2e-5, 2e-5*max|ref|), cosine > 0.999999; ints exact).
"""
import numpy as np
import pytest

import oracle
from tests.conftest import assert_fast_close, assert_fixture_close, golden_cases, load_golden
from tests.glue_fixtures import GLUE_CASES

pytestmark = pytest.mark.gpu

b2m = pytest.importorskip("onnx_runtime_dart_b200")
from onnx_runtime_dart_b200 import ops  # noqa: E402
from onnx_runtime_dart_b200.dispatch import GpuDispatch  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = b2m.Context(0)
    yield c
    c.synchronize()


def bits_equal(a, b):
    a = np.asarray(a)
    b = np.asarray(b)
    assert a.shape == b.shape, (a.shape, b.shape)
    if a.dtype.kind == "f":
        # value equality (+0 == -0), NaN-aware
        np.testing.assert_array_equal(a, b)
    else:
        np.testing.assert_array_equal(a.astype(np.int64), b.astype(np.int64))


# ---------------------------------------------------------------------------
# Golden fixtures through the dispatch hook
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("case", [c for c in golden_cases() if not c.startswith("dynamic") and c not in GLUE_CASES])
@pytest.mark.parametrize("nbits_mode", [ops.MODE_EXACT, ops.MODE_FAST])
def test_golden_fixture_via_dispatch(ctx, case, nbits_mode):
    g = load_golden(case)
    names = [None if i is None else i["name"] for i in g["inputs"]]
    inits = {i["name"]: arr for i, arr in zip(g["inputs"], g["arrays"]) if i is not None and i["initializer"]}
    elem = {i["name"]: i["tensor"]["elem_type"] for i in g["inputs"] if i is not None}
    d = GpuDispatch(ctx, inits, elem, nbits_mode=nbits_mode)
    outs = d.dispatch(g["op_type"], [n or "" for n in names], g["arrays"], g["attrs"])
    got = outs[0].numpy()
    want = g["expected_arrays"][g["outputs"][0]]
    if want.dtype.kind in "iu":
        got = got.astype(np.int64)
    if g["op_type"] == "MatMulNBits" and nbits_mode == ops.MODE_FAST:
        assert_fast_close(got, want, case)
    else:
        assert_fixture_close(got, want, case)
    # and against the oracle, bitwise, for every exact path
    if g["op_type"] != "MatMulNBits" or nbits_mode == ops.MODE_EXACT:
        from tests.test_oracle_golden import run_oracle
        bits_equal(got, run_oracle(g))


# ---------------------------------------------------------------------------
# fp32 MatMul / Gemm, EXACT
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("m", range(1, 7))
def test_matmul_small_shapes_bitwise(ctx, m):
    # every m,k,n in 1..6 (the reference's exhaustive kernel sweep)
    rng = np.random.default_rng(11 + m)
    for k in range(1, 7):
        for n in range(1, 7):
            a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
            b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
            bits_equal(ops.opMatMul(a, b, ctx=ctx).numpy(), oracle.matmul(a, b))


@pytest.mark.parametrize("mkn", [(1, 384, 384), (33, 65, 17), (7, 128, 5), (128, 64, 128), (5, 1, 9),
                                 (64, 384, 1), (1, 40, 151), (1, 128, 19), (1, 896, 512), (2, 77, 13),
                                 (3, 300, 35), (130, 257, 70)])
def test_matmul_odd_shapes_bitwise(ctx, mkn):
    m, k, n = mkn
    rng = np.random.default_rng(sum(mkn))
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    bits_equal(ops.opMatMul(a, b, ctx=ctx).numpy(), oracle.matmul(a, b))


@pytest.mark.parametrize("mkn", [(1024, 96, 1280), (640, 130, 1000)])
def test_matmul_large_tiles_bitwise(ctx, mkn):
    # Grids large enough for the 64 x 64 tile kernel (the small-tile kernel
    # serves underfilled grids such as config 1).
    m, k, n = mkn
    rng = np.random.default_rng(sum(mkn))
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    bits_equal(ops.opMatMul(a, b, ctx=ctx).numpy(), oracle.matmul(a, b, nthreads=8))


@pytest.mark.parametrize("ash,bsh", [
    ((2, 3, 5, 7), (2, 3, 7, 4)),     # fixture matmul_batched
    ((4, 1, 3), (3, 6)),              # shared 2-D B collapse: m=1 rows -> one m=4 GEMM
    ((3, 2, 5), (5, 7)),              # collapse with n % 4 != 0
    ((2, 1, 3, 5), (1, 4, 5, 2)),     # two-sided broadcast
    ((1, 2, 6), (3, 6, 3)),           # A broadcast, m < 4 tails
    ((32, 12, 16, 8), (32, 12, 8, 16)),  # attention-shaped batch
])
def test_matmul_batched_broadcast_bitwise(ctx, ash, bsh):
    rng = np.random.default_rng(len(ash) * 7 + sum(bsh))
    a = rng.standard_normal(ash).astype(np.float32)
    b = rng.standard_normal(bsh).astype(np.float32)
    got = ops.opMatMul(a, b, ctx=ctx).numpy()
    bits_equal(got, oracle.matmul(a, b))


def test_matmul_config1_bitwise_with_prepack(ctx):
    # A[128,384] x B[384,1536], B an initializer (prepacked)
    rng = np.random.default_rng(0)
    a = rng.standard_normal((128, 384)).astype(np.float32)
    b = (rng.standard_normal((384, 1536)) / np.sqrt(384)).astype(np.float32)
    w = ctx.prepack_f32(b)
    want = oracle.matmul(a, b, nthreads=8)
    bits_equal(ops.opMatMul(a, w, ctx=ctx).numpy(), want)
    bits_equal(ops.opMatMul(a, b, ctx=ctx).numpy(), want)


@pytest.mark.parametrize("mkn", [(128, 384, 1536), (1, 64, 100), (300, 200, 130), (700, 96, 2048),
                                 (1300, 64, 1792), (5, 7, 33), (4096, 256, 1280), (4100, 130, 1300),
                                 (4096, 64, 3072), (4736, 96, 512), (1280, 80, 640)])
def test_matmul_fast_tensor_core(ctx, mkn):
    # FAST mode with a prepacked weight: three bf16 products on tcgen05,
    # against the exact reference within the fast-mode tolerance (column tiles
    # 32/64/128/192/256 by the launcher's cost model, K and N tails, rows beyond
    # a 128-row tile, more tiles than SMs so each persistent CTA runs several
    # with both accumulators).
    m, k, n = mkn
    rng = np.random.default_rng(11 * m + k + n)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = (rng.standard_normal((k, n)) / np.sqrt(k)).astype(np.float32)
    w = ctx.prepack_f32(b)
    got = ops.opMatMul(a, w, mode=ops.MODE_FAST, ctx=ctx).numpy()
    want = oracle.matmul(a, b, nthreads=8)
    assert_fast_close(got, want, f"fast matmul {mkn}")
    # The split keeps ~16 mantissa bits per operand: far inside the contract.
    # A missing correction product would show up here as ~1e-3.
    assert_fast_close(got, want, f"fast matmul {mkn} (split accuracy)", max_rel=5e-5)


def test_matmul_fast_batched_shared_weight(ctx):
    rng = np.random.default_rng(12)
    a = rng.standard_normal((2, 3, 50, 64)).astype(np.float32)
    b = rng.standard_normal((64, 40)).astype(np.float32)
    w = ctx.prepack_f32(b)
    got = ops.opMatMul(a, w, mode=ops.MODE_FAST, ctx=ctx).numpy()
    assert got.shape == (2, 3, 50, 40)
    assert_fast_close(got, oracle.matmul(a, b), "fast batched matmul")


@pytest.mark.parametrize("alpha,beta,cshape", [(1.0, 1.0, (96,)), (0.5, 2.0, (200, 96)), (-1.5, 1.0, (200, 1)),
                                               (2.0, 3.0, ()), (1.0, 1.0, None)])
def test_gemm_fast_tensor_core(ctx, alpha, beta, cshape):
    rng = np.random.default_rng(13)
    M, K, N = 200, 72, 96
    a = rng.standard_normal((M, K)).astype(np.float32)
    bt = rng.standard_normal((N, K)).astype(np.float32)  # transB initializer
    c = None if cshape is None else rng.standard_normal(cshape).astype(np.float32)
    w = ctx.prepack_f32(bt, trans=True)
    got = ops.opGemm(a, w, c, alpha=alpha, beta=beta, mode=ops.MODE_FAST, ctx=ctx).numpy()
    want = oracle.gemm(a, bt, c, alpha=alpha, beta=beta, transB=True)
    assert_fast_close(got, want, f"fast gemm alpha={alpha} beta={beta} c={cshape}")


@pytest.mark.parametrize("ta,tb,alpha,beta,cshape", [
    (False, True, 1.0, 1.0, (6,)),
    (False, False, 0.5, 2.0, (1, 6)),
    (True, False, 1.0, 0.25, (4, 6)),
    (True, True, -1.5, 1.0, (4, 1)),
    (False, True, 2.0, 3.0, ()),
    (False, False, 1.0, 1.0, None),
    (False, True, 0.3, 1.0, (2, 6)),  # invalid broadcast -> ArgumentError below
])
def test_gemm_variants_bitwise(ctx, ta, tb, alpha, beta, cshape):
    rng = np.random.default_rng(3)
    M, K, N = 4, 8, 6
    a = rng.standard_normal((K, M) if ta else (M, K)).astype(np.float32)
    b = rng.standard_normal((N, K) if tb else (K, N)).astype(np.float32)
    c = None if cshape is None else rng.standard_normal(cshape).astype(np.float32)
    if cshape == (2, 6):
        with pytest.raises(b2m.ArgumentError):
            ops.opGemm(a, b, c, alpha=alpha, beta=beta, transA=ta, transB=tb, ctx=ctx)
        return
    got = ops.opGemm(a, b, c, alpha=alpha, beta=beta, transA=ta, transB=tb, ctx=ctx).numpy()
    bits_equal(got, oracle.gemm(a, b, c, alpha=alpha, beta=beta, transA=ta, transB=tb))


def test_gemm_prepack_known_answer_and_stable(ctx):
    # test/gemm_prepack_test.dart:15-55 through the dispatch hook, run twice
    w = np.arange(1, 13, dtype=np.float32).reshape(4, 3)
    c = np.array([10, 20, 30, 40], np.float32)
    x = np.arange(1, 7, dtype=np.float32).reshape(2, 3)
    d = GpuDispatch(ctx, {"W": w, "C": c})
    for _ in range(2):
        y = d.dispatch("Gemm", ["X", "W", "C"], [x, w, c], {"transB": 1})[0].numpy()
        assert y.ravel().tolist() == [24.0, 52.0, 80.0, 108.0, 42.0, 97.0, 152.0, 207.0]


def test_gemm_bert_ffn_shape_bitwise(ctx):
    rng = np.random.default_rng(7)
    a = rng.standard_normal((256, 768)).astype(np.float32)
    w = (rng.standard_normal((3072, 768)) / 28).astype(np.float32)
    c = rng.standard_normal((3072,)).astype(np.float32)
    pw = ctx.prepack_f32(w, trans=True)
    got = ops.opGemm(a, pw, c, ctx=ctx).numpy()
    bits_equal(got, oracle.gemm(a, w, c, transB=True, nthreads=8))


# ---------------------------------------------------------------------------
# MatMulInteger / QLinearMatMul
# ---------------------------------------------------------------------------

def _int_case(rng, m, k, n, adt=np.uint8, bdt=np.int8):
    lo_a, hi_a = (0, 256) if adt == np.uint8 else (-128, 128)
    lo_b, hi_b = (0, 256) if bdt == np.uint8 else (-128, 128)
    a = rng.integers(lo_a, hi_a, (m, k)).astype(adt)
    b = rng.integers(lo_b, hi_b, (k, n)).astype(bdt)
    return a, b


@pytest.mark.parametrize("m", [1, 64, 512])
def test_matmul_integer_config2_bitwise(ctx, m):
    # A u8[M,1024], aZp=128, B i8[1024,3072], per-col bZp in [-4,4]
    rng = np.random.default_rng(100 + m)
    a = rng.integers(0, 256, (m, 1024)).astype(np.uint8)
    b = rng.integers(-127, 128, (1024, 3072)).astype(np.int8)
    az = np.array(128, np.uint8)
    bz = rng.integers(-4, 5, (3072,)).astype(np.int8)
    w = ctx.prepack_i8(b)
    got = ops.opMatMulInteger(a, w, az, bz, ctx=ctx).numpy()
    bits_equal(got, oracle.matmul_integer(a, b, az, bz, nthreads=8))


@pytest.mark.parametrize("adt,bdt", [(np.uint8, np.int8), (np.uint8, np.uint8), (np.int8, np.int8),
                                     (np.int8, np.uint8)])
@pytest.mark.parametrize("zp", ["none", "scalar", "row_col"])
def test_matmul_integer_dtypes_zero_points(ctx, adt, bdt, zp):
    rng = np.random.default_rng(5)
    m, k, n = 37, 70, 45
    a, b = _int_case(rng, m, k, n, adt, bdt)
    az = bz = None
    if zp == "scalar":
        az = np.array(rng.integers(0, 100), adt)
        bz = np.array(rng.integers(0, 100), bdt)
    elif zp == "row_col":
        az = rng.integers(0, 100, (m,)).astype(adt)
        bz = rng.integers(0, 100, (n,)).astype(bdt)
    got = ops.opMatMulInteger(a, b, az, bz, ctx=ctx).numpy()
    bits_equal(got, oracle.matmul_integer(a, b, az, bz))


def test_matmul_integer_batched_and_broadcast(ctx):
    rng = np.random.default_rng(9)
    a = rng.integers(0, 256, (3, 5, 40)).astype(np.uint8)
    b = rng.integers(-128, 128, (3, 40, 9)).astype(np.int8)
    az = np.array(100, np.uint8)
    bits_equal(ops.opMatMulInteger(a, b, az, None, ctx=ctx).numpy(), oracle.matmul_integer(a, b, az, None))
    b1 = rng.integers(-128, 128, (40, 9)).astype(np.int8)
    bits_equal(ops.opMatMulInteger(a, b1, az, None, ctx=ctx).numpy(), oracle.matmul_integer(a, b1, az, None))


def test_matmul_integer_compact_known_answer(ctx):
    a = np.array([[10, 130, 250]], np.uint8)
    b = np.array([-1, 2, 3, -4, 5, 6], np.int8).reshape(3, 2)
    y = ops.opMatMulInteger(a, b, np.array(10, np.uint8), np.array(1, np.int8), ctx=ctx)
    assert ops.as_reference_int64(y).ravel().tolist() == [1200, 600]


def test_matmul_integer_bad_zero_point_is_unsupported(ctx):
    a = np.zeros((4, 6), np.uint8)
    b = np.zeros((6, 5), np.int8)
    with pytest.raises(b2m.UnsupportedError):
        ops.opMatMulInteger(a, b, np.zeros(3, np.uint8), None, ctx=ctx)


@pytest.mark.parametrize("out_int8", [False, True])
@pytest.mark.parametrize("m", [1, 4, 64])
def test_qlinear_matmul_bitwise(ctx, out_int8, m):
    rng = np.random.default_rng(m + 10 * out_int8)
    k, n = 96, 80
    a = rng.integers(0, 256, (m, k)).astype(np.uint8)
    b = rng.integers(0, 256, (k, n)).astype(np.uint8)
    a_s, b_s, y_s = np.float32(0.02), np.float32(0.05), np.float32(0.37 if out_int8 else 0.9)
    az, bz = np.array(113, np.uint8), np.array(128, np.uint8)
    lo, hi = (-128, 127) if out_int8 else (0, 255)
    yz = np.array(3, np.int8) if out_int8 else np.array(100, np.uint8)
    got = ops.opQLinearMatMul(a, a_s, az, b, b_s, bz, y_s, yz, lo=lo, hi=hi, ctx=ctx).numpy()
    assert got.dtype == (np.int8 if out_int8 else np.uint8)
    bits_equal(got, oracle.qlinear_matmul(a, a_s, az, b, b_s, bz, y_s, yz, lo, hi))


@pytest.mark.parametrize("adt,bdt", [(np.uint8, np.int8), (np.uint8, np.uint8), (np.int8, np.int8),
                                     (np.int8, np.uint8)])
@pytest.mark.parametrize("zp", ["none", "scalar", "row_col"])
@pytest.mark.parametrize("m,k,n", [(1, 1024, 300), (7, 208, 130), (16, 70, 45), (17, 1024, 200),
                                   (100, 208, 257), (300, 512, 640)])
def test_matmul_integer_packed_tensor_core(ctx, adt, bdt, zp, m, k, n):
    # Prepacked weights: M <= 16 runs the dp4a GEMV, larger M the tcgen05
    # kind::i8 kernel (K % 16 == 0; K=70 exercises the fallback), with K
    # tails inside a 128-k chunk and partial column / token tiles.
    rng = np.random.default_rng(m * 7919 + k * 31 + n)
    a, b = _int_case(rng, m, k, n, adt, bdt)
    az = bz = None
    if zp == "scalar":
        az = np.array(rng.integers(0, 100), adt)
        bz = np.array(rng.integers(0, 100), bdt)
    elif zp == "row_col":
        az = rng.integers(0, 100, (m,)).astype(adt)
        bz = rng.integers(0, 100, (n,)).astype(bdt)
    w = ctx.prepack_i8(b)
    got = ops.opMatMulInteger(a, w, az, bz, ctx=ctx).numpy()
    bits_equal(got, oracle.matmul_integer(a, b, az, bz, nthreads=8))


@pytest.mark.parametrize("out_int8", [False, True])
@pytest.mark.parametrize("m", [1, 9, 64, 200])
def test_qlinear_matmul_packed_bitwise(ctx, out_int8, m):
    rng = np.random.default_rng(500 + m + 10 * out_int8)
    k, n = 256, 384
    a = rng.integers(0, 256, (m, k)).astype(np.uint8)
    b = rng.integers(-128, 128, (k, n)).astype(np.int8)
    a_s, b_s, y_s = np.float32(0.02), np.float32(0.05), np.float32(3.7 if out_int8 else 9.0)
    az, bz = np.array(113, np.uint8), np.array(-3, np.int8)
    lo, hi = (-128, 127) if out_int8 else (0, 255)
    yz = np.array(3, np.int8) if out_int8 else np.array(100, np.uint8)
    w = ctx.prepack_i8(b)
    got = ops.opQLinearMatMul(a, a_s, az, w, b_s, bz, y_s, yz, lo=lo, hi=hi, ctx=ctx).numpy()
    bits_equal(got, oracle.qlinear_matmul(a, a_s, az, b, b_s, bz, y_s, yz, lo, hi))


def test_qlinear_per_channel_scale_unsupported(ctx):
    a = np.zeros((2, 3), np.uint8)
    b = np.zeros((3, 2), np.uint8)
    with pytest.raises(b2m.UnsupportedError):
        ops.opQLinearMatMul(a, np.float32(1), None, b, np.ones(2, np.float32), None, np.float32(1), None,
                            lo=0, hi=255, ctx=ctx)


# ---------------------------------------------------------------------------
# MatMulNBits
# ---------------------------------------------------------------------------

def nbits_case(rng, m, k, n, block=32, zp="packed", scale_sigma=0.02):
    nb = (k + block - 1) // block
    bq = rng.integers(0, 256, (n, nb, block // 2), dtype=np.uint8)
    sc = (np.abs(rng.normal(0, scale_sigma, (n, nb))) + 1e-3).astype(np.float32)
    if zp == "packed":
        z = rng.integers(0, 256, (n, (nb + 1) // 2), dtype=np.uint8)
    elif zp == "float":
        z = (rng.standard_normal((n, nb)) + 8).astype(np.float32)
    else:
        z = None
    a = rng.standard_normal((m, k)).astype(np.float32)
    return a, bq, sc, z


@pytest.mark.parametrize("m", [1, 2, 3, 4, 5, 8, 9, 33, 64, 65, 130])
@pytest.mark.parametrize("kbz", [(35, 16, "packed"), (40, 32, None), (64, 32, "float"), (300, 64, "packed"),
                                 (1024, 32, "packed"), (512, 128, None)])
def test_nbits_exact_bitwise_and_fast_close(ctx, m, kbz):
    k, block, zp = kbz
    n = 45
    rng = np.random.default_rng(m * 1000 + k + block)
    a, bq, sc, z = nbits_case(rng, m, k, n, block, zp)
    bias = rng.standard_normal((n,)).astype(np.float32) if m % 2 else None
    want = oracle.matmul_nbits(a, bq, sc, z, k, n, block, bias=bias)
    w = ops.prepack_nbits(ctx, bq, sc, z, k=k, n=n, bits=4, blockSize=block)
    exact = ops.opMatMulNBits(a, w, k=k, n=n, blockSize=block, bias=bias, mode=ops.MODE_EXACT, ctx=ctx).numpy()
    bits_equal(exact, want)
    fast = ops.opMatMulNBits(a, w, k=k, n=n, blockSize=block, bias=bias, mode=ops.MODE_FAST, ctx=ctx).numpy()
    assert_fast_close(fast, want, f"m={m} k={k} block={block} zp={zp}")


@pytest.mark.parametrize("m", [1, 8, 512])
def test_nbits_config3(ctx, m):
    # K=1024, N=3072, block 32, packed zp, scales |N(0,.02)|+1e-3
    rng = np.random.default_rng(3000 + m)
    a, bq, sc, z = nbits_case(rng, m, 1024, 3072, 32, "packed")
    want = oracle.matmul_nbits(a, bq, sc, z, 1024, 3072, 32, nthreads=8)
    w = ops.prepack_nbits(ctx, bq, sc, z, k=1024, n=3072, bits=4, blockSize=32)
    fast = ops.opMatMulNBits(a, w, k=1024, n=3072, blockSize=32, ctx=ctx).numpy()
    assert_fast_close(fast, want, f"config3 m={m}")
    exact = ops.opMatMulNBits(a, w, k=1024, n=3072, blockSize=32, mode=ops.MODE_EXACT, ctx=ctx).numpy()
    bits_equal(exact, want)


@pytest.mark.parametrize("m,n", [(416, 6400), (288, 6400), (224, 6400), (512, 3072), (200, 300)])
def test_nbits_prefill_token_tiles(ctx, m, n):
    # Shapes that select each prefill token-tile width (256, 192, 128, 96
    # tokens on a 148-SM part), partial token tiles and a partial weight-column
    # tile.
    rng = np.random.default_rng(7000 + m + n)
    a, bq, sc, z = nbits_case(rng, m, 1024, n, 32, "packed")
    bias = rng.standard_normal((n,)).astype(np.float32)
    want = oracle.matmul_nbits(a, bq, sc, z, 1024, n, 32, bias=bias, nthreads=8)
    w = ops.prepack_nbits(ctx, bq, sc, z, k=1024, n=n, bits=4, blockSize=32)
    fast = ops.opMatMulNBits(a, w, k=1024, n=n, blockSize=32, bias=bias, ctx=ctx).numpy()
    assert_fast_close(fast, want, f"prefill m={m} n={n}")


@pytest.mark.parametrize("m,k,n", [(64, 2048, 1024), (64, 3072, 1024), (64, 1024, 4096), (64, 1024, 6144),
                                   (33, 1000, 1100), (100, 4096, 256), (40, 256, 640), (96, 512, 1030),
                                   (17, 1024, 4096), (24, 1024, 6144), (32, 1024, 4100)])
def test_nbits_prefill_small_grids(ctx, m, k, n):
    # Tensor-core shapes whose grids underfill the SMs: decoder projections at
    # 64 sequences (o / down / qkv / gate_up), a K tail with a partial column
    # tile, long K on two column tiles, and the 17-32 row calls on wide
    # weights that leave the GEMV for the tensor cores; repeated calls are
    # bitwise stable.
    rng = np.random.default_rng(9000 + m + k + n)
    a, bq, sc, z = nbits_case(rng, m, k, n, 32, "packed")
    bias = rng.standard_normal((n,)).astype(np.float32)
    want = oracle.matmul_nbits(a, bq, sc, z, k, n, 32, bias=bias, nthreads=8)
    w = ops.prepack_nbits(ctx, bq, sc, z, k=k, n=n, bits=4, blockSize=32)
    first = ops.opMatMulNBits(a, w, k=k, n=n, blockSize=32, bias=bias, ctx=ctx).numpy()
    assert_fast_close(first, want, f"small grid m={m} k={k} n={n}")
    for _ in range(2):
        again = ops.opMatMulNBits(a, w, k=k, n=n, blockSize=32, bias=bias, ctx=ctx).numpy()
        bits_equal(again, first)


def test_nbits_batched_leading_dims_and_empty(ctx):
    rng = np.random.default_rng(1)
    a, bq, sc, z = nbits_case(rng, 6, 64, 24)
    a3 = a.reshape(2, 3, 64)
    got = ops.opMatMulNBits(a3, bq, sc, z, k=64, n=24, blockSize=32, mode=ops.MODE_EXACT, ctx=ctx).numpy()
    assert got.shape == (2, 3, 24)
    bits_equal(got, oracle.matmul_nbits(a3, bq, sc, z, 64, 24, 32))
    empty = np.zeros((0, 64), np.float32)
    y = ops.opMatMulNBits(empty, bq, sc, z, k=64, n=24, blockSize=32, ctx=ctx)
    assert y.shape == [0, 24]


def test_nbits_errors_mirror_reference(ctx):
    rng = np.random.default_rng(2)
    a, bq, sc, z = nbits_case(rng, 2, 64, 8)
    with pytest.raises(b2m.UnsupportedError):
        ops.opMatMulNBits(a, bq, sc, z, k=64, n=8, bits=3, blockSize=32, ctx=ctx)
    with pytest.raises(b2m.ArgumentError, match="invalid K, N, block_size"):
        ops.opMatMulNBits(a, bq, sc, z, k=64, n=8, blockSize=24, ctx=ctx)
    with pytest.raises(b2m.ArgumentError, match="invalid packed weights or scales"):
        ops.opMatMulNBits(a, bq[:, :1], sc, z, k=64, n=8, blockSize=32, ctx=ctx)
    with pytest.raises(b2m.ArgumentError, match="invalid zero_points"):
        ops.opMatMulNBits(a, bq, sc, z[:4], k=64, n=8, blockSize=32, ctx=ctx)
    with pytest.raises(b2m.ArgumentError, match="bias must be floating point"):
        ops.opMatMulNBits(a, bq, sc, z, k=64, n=8, blockSize=32, bias=np.zeros(7, np.float32), ctx=ctx)
    d = GpuDispatch(ctx, {"B": bq, "S": sc})
    with pytest.raises(b2m.UnsupportedError, match="g_idx"):
        d.dispatch("MatMulNBits", ["A", "B", "S", "", "G"], [a, bq, sc, None, np.zeros(64)],
                   {"K": 64, "N": 8, "block_size": 32})


def test_nbits_host_and_dev_entry_points_match(ctx):
    import ctypes

    import torch
    rng = np.random.default_rng(4)
    a, bq, sc, z = nbits_case(rng, 8, 1024, 3072)
    bias = rng.standard_normal((3072,)).astype(np.float32)
    w = ops.prepack_nbits(ctx, bq, sc, z, k=1024, n=3072, bits=4, blockSize=32)
    ref = ops.opMatMulNBits(a, w, k=1024, n=3072, blockSize=32, bias=bias, ctx=ctx).numpy()
    yh = np.empty((8, 3072), np.float32)
    b2m._native.check(ctx.lib.b2m_matmul_nbits_host(ctx.handle, a.ctypes.data_as(ctypes.c_void_p), 8, w.handle,
                                                    bias.ctypes.data_as(ctypes.c_void_p), ops.MODE_FAST,
                                                    yh.ctypes.data_as(ctypes.c_void_p)))
    bits_equal(yh, ref)
    ta = torch.from_numpy(a).cuda()
    tb = torch.from_numpy(bias).cuda()
    ty = torch.empty((8, 3072), device="cuda")
    torch.cuda.synchronize()
    ctx.set_stream(torch.cuda.current_stream().cuda_stream)
    b2m._native.check(ctx.lib.b2m_matmul_nbits_dev(ctx.handle, ctypes.c_void_p(ta.data_ptr()), 8, w.handle,
                                                   ctypes.c_void_p(tb.data_ptr()), ops.MODE_FAST,
                                                   ctypes.c_void_p(ty.data_ptr())))
    torch.cuda.synchronize()
    ctx.set_stream(None)
    bits_equal(ty.cpu().numpy(), ref)


def test_output_reuse_and_control(ctx):
    rng = np.random.default_rng(8)
    a = rng.standard_normal((16, 32)).astype(np.float32)
    b = rng.standard_normal((32, 8)).astype(np.float32)
    out = ctx.empty((16, 8))
    y = ops.opMatMul(a, b, ctx=ctx, out=out)
    assert y is out
    bits_equal(out.numpy(), oracle.matmul(a, b))
    with pytest.raises(b2m.ArgumentError):
        ops.opMatMul(a, b, ctx=ctx, out=ctx.empty((16, 9)))
    c2 = b2m.Context(0)
    c2.enable_cancel_flag()
    c2.cancel(True)
    with pytest.raises(b2m.OnnxCancelledException):
        ops.opMatMul(a, b, ctx=c2)
    c2.cancel(False)
    c2.set_byte_budget(100)
    with pytest.raises(b2m.OnnxMemoryLimitException):
        ops.opMatMul(a, b, ctx=c2)
    c2.close()
