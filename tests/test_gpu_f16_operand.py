"""GPU tests of the producer-written f16 operand of FAST MatMulNBits.

Where a FAST MatMulNBits call takes the tensor-core route, the GEMM first
rounds its fp32 activations to f16 in a conversion launch. In a chain the op
that produces those activations (RMSNorm, SiLU*Mul) can write the f16 copy
itself, and b2m_matmul_nbits_f16_dev takes it: one launch fewer per
projection and the same bits. The tests hold every piece to bit equality with
the path it replaces: the route query, the f16 entry against the fp32 entry,
the producers' f16 copies against rounding their fp32 outputs, and a decoder
(Qwen3-0.6B shapes, two layers) with and without producer-written operands.
The reference runs these ops as separate Dart kernels in fp32
(lib/src/onnx_qlinear_ops.dart:115-228, lib/src/onnx_ops.dart:1771); FAST mode
is held to its tolerance contract elsewhere."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import onnx_runtime_dart_b200 as b2m  # noqa: E402
from onnx_runtime_dart_b200 import _native as N  # noqa: E402
from onnx_runtime_dart_b200.decoder import DecoderConfig, Int4Decoder  # noqa: E402


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


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


def _route(ctx, w, m, mode):
    r = ctypes.c_int32(-1)
    N.check(ctx.lib.b2m_matmul_nbits_route(ctx.handle, w.handle, m, mode, ctypes.byref(r)))
    return r.value


def test_route_query(ctx):
    w = _weight(ctx, np.random.default_rng(0), 1024, 3072)
    assert _route(ctx, w, 1, N.MODE_FAST) == N.ROUTE_GEMV
    assert _route(ctx, w, 8, N.MODE_FAST) == N.ROUTE_GEMV
    assert _route(ctx, w, 512, N.MODE_FAST) == N.ROUTE_TC_F16
    assert _route(ctx, w, 1, N.MODE_PRECISE) == N.ROUTE_GEMV
    assert _route(ctx, w, 512, N.MODE_EXACT) == N.ROUTE_OTHER
    assert _route(ctx, w, 0, N.MODE_FAST) == N.ROUTE_OTHER
    w.free()


@pytest.mark.parametrize("m,k,n", [(64, 1024, 4096), (512, 1024, 3072), (777, 3072, 1024)])
def test_f16_entry_matches_fast_entry_bitwise(ctx, m, k, n):
    rng = np.random.default_rng(m)
    w = _weight(ctx, rng, k, n)
    lib, h = ctx.lib, ctx.handle
    a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    a16 = a.half()  # round to nearest, as the GEMM's conversion rounds
    bias = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()
    y32 = torch.full((m, n), float("nan"), device="cuda")
    y16 = torch.full((m, n), float("nan"), device="cuda")
    torch.cuda.synchronize()
    N.check(lib.b2m_matmul_nbits_dev(h, _p(a), m, w.handle, _p(bias), N.MODE_FAST, _p(y32)))
    N.check(lib.b2m_matmul_nbits_f16_dev(h, _p(a16), m, w.handle, _p(bias), _p(y16)))
    N.check(lib.b2m_synchronize(h))
    np.testing.assert_array_equal(y16.cpu().numpy(), y32.cpu().numpy())
    # a row count the GEMV serves is refused
    assert lib.b2m_matmul_nbits_f16_dev(h, _p(a16), 1, w.handle, None, _p(y16)) == N.B2M_ERR_UNSUPPORTED
    w.free()


@pytest.mark.parametrize("rows,d,skip", [(64, 1024, True), (4096, 1024, False), (3, 3072, True)])
def test_rmsnorm_f16_copy(ctx, rows, d, skip):
    rng = np.random.default_rng(rows + d)
    lib, h = ctx.lib, ctx.handle
    x = torch.from_numpy(rng.standard_normal((rows, d)).astype(np.float32)).cuda()
    s = torch.from_numpy(rng.standard_normal((rows, d)).astype(np.float32)).cuda() if skip else None
    g = torch.from_numpy(rng.standard_normal(d).astype(np.float32)).cuda()
    y_ref, y, sum_ref, sum_out = (torch.empty((rows, d), device="cuda") for _ in range(4))
    y16 = torch.empty((rows, d), device="cuda", dtype=torch.float16)
    torch.cuda.synchronize()
    N.check(lib.b2m_rmsnorm_dev(h, _p(x), _p(s) if skip else None, _p(g), _p(y_ref), _p(sum_ref) if skip else None,
                                rows, d, 1e-6))
    N.check(lib.b2m_rmsnorm_f16_dev(h, _p(x), _p(s) if skip else None, _p(g), _p(y), _p(sum_out) if skip else None,
                                    _p(y16), rows, d, 1e-6))
    N.check(lib.b2m_synchronize(h))
    assert torch.equal(y, y_ref)
    assert torch.equal(y16, y_ref.half())
    if skip:
        assert torch.equal(sum_out, sum_ref)
    # Only the f16 rows (the projection's operand): the same bits, the same sum.
    y16b = torch.zeros((rows, d), device="cuda", dtype=torch.float16)
    sum_b = torch.zeros((rows, d), device="cuda")
    torch.cuda.synchronize()
    N.check(lib.b2m_rmsnorm_f16_dev(h, _p(x), _p(s) if skip else None, _p(g), None, _p(sum_b) if skip else None,
                                    _p(y16b), rows, d, 1e-6))
    N.check(lib.b2m_synchronize(h))
    assert torch.equal(y16b, y16)
    if skip:
        assert torch.equal(sum_b, sum_ref)


def test_rmsnorm_f16_without_fp32_rows_needs_aligned_rows(ctx):
    """y = NULL is refused where only the scalar kernel serves the layout."""
    lib, h = ctx.lib, ctx.handle
    x = torch.zeros((4, 1026), device="cuda")  # rows of 1024 from offset 2: 8-byte aligned only
    g = torch.ones(1024, device="cuda")
    y16 = torch.zeros((4, 1024), device="cuda", dtype=torch.float16)
    torch.cuda.synchronize()
    with pytest.raises(N.ArgumentError, match="y may be NULL only"):
        N.check(lib.b2m_rmsnorm_f16_dev(h, ctypes.c_void_p(x.data_ptr() + 8), None, _p(g), None, None, _p(y16), 4,
                                        1024, 1e-6))


@pytest.mark.parametrize("rows,d", [(64, 3072), (2048, 3072)])
def test_silu_mul_f16_copy(ctx, rows, d):
    rng = np.random.default_rng(rows)
    lib, h = ctx.lib, ctx.handle
    gu = torch.from_numpy(rng.standard_normal((rows, 2 * d)).astype(np.float32)).cuda()
    y_ref, y = torch.empty((rows, d), device="cuda"), torch.empty((rows, d), device="cuda")
    y16 = torch.empty((rows, d), device="cuda", dtype=torch.float16)
    up = ctypes.c_void_p(gu.data_ptr() + d * 4)
    torch.cuda.synchronize()
    N.check(lib.b2m_silu_mul_dev(h, _p(gu), up, 2 * d, 2 * d, _p(y_ref), rows, d))
    N.check(lib.b2m_silu_mul_f16_dev(h, _p(gu), up, 2 * d, 2 * d, _p(y), _p(y16), rows, d))
    N.check(lib.b2m_synchronize(h))
    assert torch.equal(y, y_ref)
    assert torch.equal(y16, y_ref.half())


def test_decoder_producer_f16_same_bits(ctx):
    """Qwen3-0.6B shapes, two layers, 64 sequences: a 32-token prefill (2048
    rows) and two greedy decode steps (64 rows, the tensor-core route), with
    and without the producer-written f16 operands: identical logits."""
    cfg = DecoderConfig.qwen3_0_6b()
    cfg.layers = 2
    B, S = 64, 32
    prompt = np.random.default_rng(3).integers(0, cfg.vocab, (B, S))
    out = []
    for pf in (False, True):
        dec = Int4Decoder(ctx, cfg, batch=B, cap=S + 4, max_prefill=S, seed=11, producer_f16=pf)
        dec.prefill(prompt)
        torch.cuda.synchronize()
        logits = [dec.logits.cpu().numpy().copy()]
        dec.decode(2)
        torch.cuda.synchronize()
        logits.append(dec.logits.cpu().numpy().copy())
        out.append(logits)
        del dec
    for a, b in zip(out[0], out[1]):
        np.testing.assert_array_equal(a, b)


# --- the FAST fp32 Gemm's bf16 hi / lo planes written by their producer ---

from onnx_runtime_dart_b200.bert import BertConfig, BertEncoder  # noqa: E402


def _gemm_fast(ctx, a, m, k, w, bias, y):
    """b2m_gemm_f32 FAST, alpha = beta = 1, C = bias (a BERT Gemm)."""
    at = ctx.wrap(a.data_ptr(), (m, k), np.float32)
    bt = ctx.wrap(bias.data_ptr(), (bias.numel(),), np.float32)
    yt = ctx.wrap(y.data_ptr(), tuple(y.shape), np.float32)  # kept alive across the call
    yh = ctypes.c_void_p(yt.handle.value)
    N.check(ctx.lib.b2m_gemm_f32(ctx.handle, at.handle, None, w.handle, bt.handle, ctypes.c_float(1.0),
                                 ctypes.c_float(1.0), 0, 0, N.MODE_FAST, ctypes.byref(yh)))
    N.check(ctx.lib.b2m_synchronize(ctx.handle))


@pytest.mark.parametrize("rows", [128, 4096])
def test_layernorm_and_gelu_planes_feed_the_gemm_bitwise(ctx, rows):
    rng = np.random.default_rng(rows)
    lib, h = ctx.lib, ctx.handle
    d, n, i = 768, 3072, 3072
    x = torch.from_numpy(rng.standard_normal((rows, d)).astype(np.float32)).cuda()
    s = torch.from_numpy(rng.standard_normal((rows, d)).astype(np.float32)).cuda()
    g = torch.from_numpy((1 + 0.1 * rng.standard_normal(d)).astype(np.float32)).cuda()
    b = torch.from_numpy((0.1 * rng.standard_normal(d)).astype(np.float32)).cuda()
    w1 = ctx.prepack_f32((rng.standard_normal((d, n)) / np.sqrt(d)).astype(np.float32))
    w2 = ctx.prepack_f32((rng.standard_normal((i, d)) / np.sqrt(i)).astype(np.float32))
    b1 = torch.from_numpy(rng.standard_normal(n).astype(np.float32)).cuda()
    b2 = torch.from_numpy(rng.standard_normal(d).astype(np.float32)).cuda()
    y_ref, y = torch.empty((rows, d), device="cuda"), torch.empty((rows, d), device="cuda")
    planes = torch.empty((2, rows, d), device="cuda", dtype=torch.bfloat16)
    torch.cuda.synchronize()
    N.check(lib.b2m_layernorm_dev(h, _p(x), _p(s), _p(g), _p(b), _p(y_ref), None, rows, d, ctypes.c_double(1e-12)))
    N.check(lib.b2m_layernorm_split_dev(h, _p(x), _p(s), _p(g), _p(b), _p(y), None, _p(planes), rows, d,
                                        ctypes.c_double(1e-12)))
    f_ref, f = torch.empty((rows, n), device="cuda"), torch.empty((rows, n), device="cuda")
    _gemm_fast(ctx, y_ref, rows, d, w1, b1, f_ref)
    N.check(lib.b2m_gemm_f32_split_dev(h, _p(planes), rows, w1.handle, _p(b1), _p(f)))
    N.check(lib.b2m_synchronize(h))
    assert torch.equal(y, y_ref)
    assert torch.equal(f, f_ref)
    # GELU: planes only, then the FFN-down Gemm
    g_ref = torch.empty_like(f_ref)
    N.check(lib.b2m_gelu_dev(h, _p(f_ref), _p(g_ref), rows * n))
    gplanes = torch.empty((2, rows, n), device="cuda", dtype=torch.bfloat16)
    N.check(lib.b2m_gelu_split_dev(h, _p(f), None, _p(gplanes), rows, n))
    o_ref, o = torch.empty((rows, d), device="cuda"), torch.empty((rows, d), device="cuda")
    _gemm_fast(ctx, g_ref, rows, i, w2, b2, o_ref)
    N.check(lib.b2m_gemm_f32_split_dev(h, _p(gplanes), rows, w2.handle, _p(b2), _p(o)))
    N.check(lib.b2m_synchronize(h))
    assert torch.equal(o, o_ref)
    w1.free()
    w2.free()


def test_bert_producer_split_same_bits(ctx):
    """BERT-base shapes, two layers, 4 x 128 tokens: the encoder with the
    producer-written planes and with the Gemms' own split pass give the same
    last hidden state."""
    cfg = BertConfig.base()
    cfg.layers = 2
    ids = np.random.default_rng(9).integers(0, cfg.vocab, (4, 128))
    outs = []
    for ps in (False, True):
        enc = BertEncoder(ctx, cfg, 4, 128, seed=21, producer_split=ps)
        assert enc.split == ps
        outs.append(enc.forward(ids, use_graph=False))
        del enc
    np.testing.assert_array_equal(outs[0], outs[1])


# --- 33..64 rows (the decode projections at 64 sequences) against the oracle ---

import oracle  # noqa: E402
from tests.conftest import assert_fast_close  # noqa: E402


@pytest.mark.parametrize("m,k,n", [(33, 1024, 384), (48, 3072, 1000), (64, 1024, 6144), (64, 2048, 1024)])
def test_33_to_64_rows_within_fast_contract(ctx, m, k, n):
    """33..64 rows (the decoder's decode projections at 64 sequences) take
    the tensor-core route: within the FAST contract of the oracle's
    opMatMulNBits (onnx_qlinear_ops.dart:208-226) through the fp32 entry,
    bit for bit the same through the f16 entry and on a second call."""
    rng = np.random.default_rng(m * 7 + n)
    nb = k // 32
    bq = rng.integers(0, 256, (n, nb, 16), dtype=np.uint8)
    sc = (np.abs(rng.normal(0, 0.02, (n, nb))) + 1e-3).astype(np.float32)
    zp = rng.integers(0, 256, (n, (nb + 1) // 2), dtype=np.uint8)
    w = ctx.prepack_nbits(bq, sc, zp, k, n, 4, 32)
    assert _route(ctx, w, m, N.MODE_FAST) == N.ROUTE_TC_F16
    lib, h = ctx.lib, ctx.handle
    a_np = rng.standard_normal((m, k)).astype(np.float32)
    bias_np = rng.standard_normal(n).astype(np.float32)
    a = torch.from_numpy(a_np).cuda()
    bias = torch.from_numpy(bias_np).cuda()
    y1, y2, y3 = (torch.full((m, n), float("nan"), device="cuda") for _ in range(3))
    torch.cuda.synchronize()
    N.check(lib.b2m_matmul_nbits_dev(h, _p(a), m, w.handle, _p(bias), N.MODE_FAST, _p(y1)))
    N.check(lib.b2m_matmul_nbits_dev(h, _p(a), m, w.handle, _p(bias), N.MODE_FAST, _p(y2)))
    N.check(lib.b2m_matmul_nbits_f16_dev(h, _p(a.half()), m, w.handle, _p(bias), _p(y3)))
    N.check(lib.b2m_synchronize(h))
    got = y1.cpu().numpy()
    np.testing.assert_array_equal(y2.cpu().numpy(), got)
    np.testing.assert_array_equal(y3.cpu().numpy(), got)
    want = oracle.matmul_nbits(a_np, bq, sc, zp, k, n, 32, bias=bias_np, nthreads=8)
    assert_fast_close(got, want, f"m={m} k={k} n={n}")
    w.free()


@pytest.mark.parametrize("b,s,past,D", [(64, 1, 300, 128), (2, 512, 0, 128), (3, 5, 7, 96)])
def test_gqa_f16_copy(ctx, b, s, past, D):
    """b2m_gqa_f16_dev: the same fp32 output as b2m_gqa_dev and its f16 copy
    equal to rounding it (decode with key splits, the tensor-core prefill, and
    a head_dim the tensor-core kernel does not take: the CUDA-core kernel plus
    a rounding pass)."""
    rng = np.random.default_rng(b * 1000 + s)
    lib, h = ctx.lib, ctx.handle
    H, KVH, cap = 16, 8, 640
    q = torch.from_numpy(rng.standard_normal((b * s, H * D)).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.standard_normal((b * s, KVH * D)).astype(np.float32)).cuda()
    v = torch.from_numpy(rng.standard_normal((b * s, KVH * D)).astype(np.float32)).cuda()
    cache0 = torch.from_numpy(rng.standard_normal((b, KVH, cap, D)).astype(np.float32)).cuda()
    half = D // 2
    inv = 1.0 / (10000.0 ** (np.arange(half) * 2.0 / D))
    ang = np.arange(cap)[:, None] * inv[None, :]
    cos = torch.from_numpy(np.cos(ang).astype(np.float32)).cuda()
    sin = torch.from_numpy(np.sin(ang).astype(np.float32)).cuda()
    outs = []
    for f16 in (False, True):
        kc, vc = cache0.clone(), cache0.clone()
        past_t = torch.full((b,), past, dtype=torch.int32, device="cuda")
        out = torch.full((b * s, H * D), float("nan"), device="cuda")
        out16 = torch.empty((b * s, H * D), device="cuda", dtype=torch.float16)
        torch.cuda.synchronize()
        args = [h, _p(q), _p(k), _p(v), H * D, KVH * D, _p(kc), _p(vc), _p(past_t), _p(cos), _p(sin), half, D, 0,
                _p(out)]
        tail = [b, s, H, KVH, D, cap, ctypes.c_float(0.0)]
        if f16:
            N.check(lib.b2m_gqa_f16_dev(*args, _p(out16), *tail))
        else:
            N.check(lib.b2m_gqa_dev(*args, *tail))
        N.check(lib.b2m_synchronize(h))
        outs.append((out, out16))
    assert torch.equal(outs[1][0], outs[0][0])
    assert torch.equal(outs[1][1], outs[0][0].half())


@pytest.mark.parametrize("b,s,heads,D", [(4, 128, 12, 64), (2, 40, 8, 96)])
def test_mha_split_planes(ctx, b, s, heads, D):
    """b2m_mha_split_dev: the same fp32 output as b2m_mha_dev and planes that
    feed the FAST Gemm to the bits of the Gemm's own split (the tensor-core MHA
    at BERT's shape, and a head_dim it does not take: a split pass after)."""
    rng = np.random.default_rng(s + heads)
    lib, h = ctx.lib, ctx.handle
    H = heads * D
    qkv = torch.from_numpy(rng.standard_normal((b * s, 3 * H)).astype(np.float32)).cuda()
    mask = torch.zeros((b, s), device="cuda")
    mask[0, s - 3:] = -10000.0
    w = ctx.prepack_f32((rng.standard_normal((H, 256)) / np.sqrt(H)).astype(np.float32))
    bias = torch.from_numpy(rng.standard_normal(256).astype(np.float32)).cuda()
    out_ref, out = torch.empty((b * s, H), device="cuda"), torch.empty((b * s, H), device="cuda")
    planes = torch.empty((2, b * s, H), device="cuda", dtype=torch.bfloat16)
    base = qkv.data_ptr()
    q_, k_, v_ = ctypes.c_void_p(base), ctypes.c_void_p(base + H * 4), ctypes.c_void_p(base + 2 * H * 4)
    torch.cuda.synchronize()
    N.check(lib.b2m_mha_dev(h, q_, k_, v_, 3 * H, 3 * H, _p(mask), s, 0, 0, _p(out_ref), b, s, s, heads, heads, D,
                            ctypes.c_float(0.0), 0))
    N.check(lib.b2m_mha_split_dev(h, q_, k_, v_, 3 * H, 3 * H, _p(mask), s, 0, 0, _p(out), _p(planes), b, s, s, heads,
                                  heads, D, ctypes.c_float(0.0), 0))
    y_ref, y = torch.empty((b * s, 256), device="cuda"), torch.empty((b * s, 256), device="cuda")
    _gemm_fast(ctx, out_ref, b * s, H, w, bias, y_ref)
    N.check(lib.b2m_gemm_f32_split_dev(h, _p(planes), b * s, w.handle, _p(bias), _p(y)))
    N.check(lib.b2m_synchronize(h))
    assert torch.equal(out, out_ref)
    assert torch.equal(y, y_ref)
    w.free()
