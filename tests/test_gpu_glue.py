"""GPU tests of the device-resident glue ops (RMSNorm, LayerNorm, SiLU*Mul,
GELU, Add, Gather, ArgMax, RotaryEmbedding, GroupQueryAttention with rotary
and a KV cache, MultiHeadAttention) through the C ABI: against the reference's
own fixtures for these ops, and against the numpy restatement in
oracle/glue.py (itself pinned to those fixtures) on larger seeded cases and on
the BERT / decoder chains."""
import ctypes

import numpy as np
import pytest

from oracle import glue
from tests import chain_refs
from tests.conftest import assert_fast_close, assert_fixture_close, load_golden
from tests.glue_fixtures import GLUE_CASES, run_case

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import onnx_runtime_dart_b200 as b2m  # noqa: E402
from onnx_runtime_dart_b200 import _native as N  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = b2m.Context(0)
    yield c
    c.synchronize()


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _close(got, want, rtol=1e-5, what=""):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    scale = max(float(np.max(np.abs(want))), 1e-30)
    err = float(np.max(np.abs(got - want))) / scale
    assert err <= rtol, f"{what}: max rel err {err:.3e} > {rtol}"


@pytest.mark.parametrize("rows,d,skip", [(7, 1024, False), (33, 128, True), (5, 100, True)])
def test_rmsnorm_matches_reference(ctx, rows, d, skip):
    rng = np.random.default_rng(rows + d)
    x = rng.standard_normal((rows, d)).astype(np.float32)
    s = rng.standard_normal((rows, d)).astype(np.float32) if skip else None
    g = (1 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    want, wsum = glue.rmsnorm(x, g, 1e-6, skip=s)
    dx, dg, dy = _d(x), _d(g), torch.empty_like(_d(x))
    ds = _d(s) if skip else None
    dsum = torch.empty_like(dx) if skip else None
    N.check(ctx.lib.b2m_rmsnorm_dev(ctx.handle, _p(dx), _p(ds), _p(dg), _p(dy), _p(dsum), rows, d, 1e-6))
    torch.cuda.synchronize()
    _close(dy.cpu().numpy(), want, 2e-7, "rmsnorm")
    if skip:
        np.testing.assert_array_equal(dsum.cpu().numpy(), wsum)


def test_rmsnorm_heads_in_place(ctx):
    rng = np.random.default_rng(3)
    tokens, heads, hd, stride = 6, 4, 32, 4 * 32 + 64
    x = rng.standard_normal((tokens, stride)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(hd)).astype(np.float32)
    want = x.copy()
    want[:, : heads * hd] = glue.rmsnorm(x[:, : heads * hd].reshape(tokens * heads, hd), g, 1e-6)[0].reshape(
        tokens, heads * hd)
    dx, dg = _d(x), _d(g)
    N.check(ctx.lib.b2m_rmsnorm_heads_dev(ctx.handle, _p(dx), _p(dg), _p(dx), tokens, heads, hd, stride, 1e-6))
    torch.cuda.synchronize()
    _close(dx.cpu().numpy(), want, 2e-7, "rmsnorm heads")


def test_layernorm_matches_reference(ctx):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((9, 768)).astype(np.float32)
    s = rng.standard_normal((9, 768)).astype(np.float32)
    g = rng.standard_normal(768).astype(np.float32)
    b = rng.standard_normal(768).astype(np.float32)
    want, _ = glue.layernorm(x, g, b, 1e-12, skip=s)
    dx, ds, dg, db = _d(x), _d(s), _d(g), _d(b)
    dy = torch.empty_like(dx)
    N.check(ctx.lib.b2m_layernorm_dev(ctx.handle, _p(dx), _p(ds), _p(dg), _p(db), _p(dy), None, 9, 768, 1e-12))
    torch.cuda.synchronize()
    _close(dy.cpu().numpy(), want, 2e-7, "layernorm")


def test_elementwise_gather_argmax(ctx):
    rng = np.random.default_rng(5)
    gu = rng.standard_normal((10, 2 * 48)).astype(np.float32)
    dgu = _d(gu)
    dy = torch.empty((10, 48), device="cuda")
    N.check(ctx.lib.b2m_silu_mul_dev(ctx.handle, _p(dgu), ctypes.c_void_p(dgu.data_ptr() + 48 * 4), 96, 96, _p(dy),
                                     10, 48))
    x = rng.standard_normal(1000).astype(np.float32)
    dx = _d(x)
    dgl = torch.empty_like(dx)
    N.check(ctx.lib.b2m_gelu_dev(ctx.handle, _p(dx), _p(dgl), 1000))
    a = rng.standard_normal((4, 8)).astype(np.float32)
    b = rng.standard_normal(8).astype(np.float32)
    da, db = _d(a), _d(b)
    dsum = torch.empty_like(da)
    N.check(ctx.lib.b2m_add_dev(ctx.handle, _p(da), _p(db), _p(dsum), 4, 8, 1))
    table = rng.standard_normal((50, 16)).astype(np.float32)
    ids = np.array([3, 0, 49, 7, 7], np.int64)
    dt, di = _d(table), _d(ids)
    drows = torch.empty((5, 16), device="cuda")
    N.check(ctx.lib.b2m_gather_rows_dev(ctx.handle, _p(dt), _p(di), _p(drows), 5, 50, 16))
    logits = rng.standard_normal((3, 151936)).astype(np.float32)
    logits[1, 77] = logits[1, 99] = 50.0  # tie: the first index wins
    dl = _d(logits)
    dam = torch.empty(3, device="cuda", dtype=torch.int64)
    N.check(ctx.lib.b2m_argmax_dev(ctx.handle, _p(dl), _p(dam), 3, 151936))
    torch.cuda.synchronize()
    _close(dy.cpu().numpy(), glue.silu_mul(gu[:, :48], gu[:, 48:]), 1e-6, "silu_mul")
    _close(dgl.cpu().numpy(), glue.gelu(x), 1e-6, "gelu")
    np.testing.assert_array_equal(dsum.cpu().numpy(), a + b)
    np.testing.assert_array_equal(drows.cpu().numpy(), table[ids])
    got = dam.cpu().numpy()
    np.testing.assert_array_equal(got, glue.argmax(logits))
    assert got[1] == 77


@pytest.mark.parametrize("b,s,past,h,kvh,d,interleaved", [(2, 5, 0, 4, 2, 32, 0), (3, 1, 9, 16, 8, 128, 0),
                                                           (1, 7, 3, 6, 3, 64, 1), (2, 40, 0, 8, 8, 96, 0),
                                                           (2, 130, 20, 4, 2, 128, 0), (1, 1, 300, 16, 2, 128, 0),
                                                           (2, 1, 0, 4, 4, 64, 1), (8, 1, 576, 16, 8, 128, 0),
                                                           (2, 1, 1000, 16, 4, 32, 0), (3, 1, 700, 8, 8, 96, 1),
                                                           (64, 1, 40, 16, 8, 128, 0), (2, 300, 0, 16, 8, 128, 0),
                                                           (1, 129, 70, 4, 1, 64, 1), (3, 64, 5, 8, 4, 128, 1)])
def test_gqa_cache_rotary(ctx, b, s, past, h, kvh, d, interleaved):
    # Prefill-shaped and decode-shaped calls; `past` positions already cached.
    rng = np.random.default_rng(b * 100 + s + past + d)
    cap = past + s + 3
    cos, sin = glue.rope_cache(cap, d // 2, 1e4)
    q = rng.standard_normal((b, s, h * d)).astype(np.float32)
    k = rng.standard_normal((b, s, kvh * d)).astype(np.float32)
    v = rng.standard_normal((b, s, kvh * d)).astype(np.float32)
    pk = rng.standard_normal((b, kvh, past, d)).astype(np.float32) if past else None
    pv = rng.standard_normal((b, kvh, past, d)).astype(np.float32) if past else None
    want, wk, wv = glue.gqa(q, k, v, h, kvh, pk, pv, cos, sin, interleaved=bool(interleaved))
    kc = np.zeros((b, kvh, cap, d), np.float32)
    vc = np.zeros((b, kvh, cap, d), np.float32)
    if past:
        kc[:, :, :past] = pk
        vc[:, :, :past] = pv
    dq, dk, dv, dkc, dvc = _d(q), _d(k), _d(v), _d(kc), _d(vc)
    dpast = _d(np.full(b, past, np.int32))
    dcos, dsin = _d(cos), _d(sin)
    dout = torch.empty_like(dq)
    N.check(ctx.lib.b2m_gqa_dev(ctx.handle, _p(dq), _p(dk), _p(dv), h * d, kvh * d, _p(dkc), _p(dvc), _p(dpast),
                                _p(dcos), _p(dsin), d // 2, d, interleaved, _p(dout), b, s, h, kvh, d, cap, 0.0))
    torch.cuda.synchronize()
    _close(dout.cpu().numpy(), want, 2e-5, "gqa out")
    _close(dkc.cpu().numpy()[:, :, : past + s], wk, 1e-6, "present key")
    np.testing.assert_array_equal(dvc.cpu().numpy()[:, :, : past + s], wv)


@pytest.mark.parametrize("b,s,t,h,kvh,d,mask_mode,causal,packed", [
    (2, 128, 128, 12, 12, 64, "pad", 0, 1),   # BERT-base shaped, fused QKV rows, padded keys
    (3, 5, 9, 4, 2, 32, "bcast", 0, 0),       # cross-attention shaped, one mask row for all batches
    (1, 70, 70, 4, 4, 128, None, 1, 1),       # causal, two query tiles
    (2, 33, 40, 2, 1, 48, "pad", 0, 0),       # head dim outside the tiled kernel's set
    (2, 1, 17, 4, 4, 64, "inf", 0, 0),        # one query, -inf masked keys
    (2, 130, 130, 8, 8, 96, None, 0, 1),      # ragged last tiles in both directions
    (2, 70, 70, 4, 4, 64, "bias4d", 0, 0),    # attention_bias [b][h][s][t], per query row
    (2, 9, 11, 4, 4, 48, "bias1h", 0, 0),     # attention_bias with one head, per-query-warp kernel
    (2, 100, 100, 4, 2, 64, None, 1, 0),      # causal, grouped kv heads, tensor-core kernel
    (3, 128, 77, 2, 2, 64, "pad", 0, 0),      # cross-attention with ragged keys, tensor-core kernel
])
def test_mha_additive_mask(ctx, b, s, t, h, kvh, d, mask_mode, causal, packed):
    rng = np.random.default_rng(b * 1000 + s * 7 + t + d)
    q = rng.standard_normal((b, s, h * d)).astype(np.float32)
    k = rng.standard_normal((b, t, kvh * d)).astype(np.float32)
    v = rng.standard_normal((b, t, kvh * d)).astype(np.float32)
    mask = None
    if mask_mode == "pad":
        mask = np.zeros((b, t), np.float32)
        for i in range(b):
            mask[i, t - 1 - i * 3:] = -10000.0     # (1 - attention_mask) * -10000
    elif mask_mode == "bcast":
        mask = np.broadcast_to(rng.standard_normal(t).astype(np.float32), (b, t)).copy()
    elif mask_mode == "inf":
        mask = np.zeros((b, t), np.float32)
        mask[:, 3::4] = -np.inf
    bias4d = None
    strides = (0 if mask_mode == "bcast" else t, 0, 0)
    if mask_mode in ("bias4d", "bias1h"):
        bh = h if mask_mode == "bias4d" else 1
        bias4d = rng.standard_normal((b, bh, s, t)).astype(np.float32)
        strides = (bh * s * t, s * t if bh > 1 else 0, t)
    want = glue.mha(q, k, v, h, kvh, mask, causal=bool(causal), bias4d=bias4d)
    if packed:
        # One [b][s][(h + 2 kvh) d] tensor as a fused QKV projection writes it.
        assert s == t
        qkv = np.concatenate([q, k, v], axis=-1)
        dqkv = _d(qkv)
        rs = qkv.shape[-1]
        base = dqkv.data_ptr()
        pq, pk, pv = (ctypes.c_void_p(base), ctypes.c_void_p(base + h * d * 4),
                      ctypes.c_void_p(base + (h + kvh) * d * 4))
        q_rs = kv_rs = rs
    else:
        dq, dk, dv = _d(q), _d(k), _d(v)
        pq, pk, pv = _p(dq), _p(dk), _p(dv)
        q_rs, kv_rs = h * d, kvh * d
    dm = _d(mask[:1] if mask_mode == "bcast" else mask) if mask is not None else None
    if bias4d is not None:
        dm = _d(bias4d)
    dout = torch.empty((b, s, h * d), dtype=torch.float32, device="cuda")
    N.check(ctx.lib.b2m_mha_dev(ctx.handle, pq, pk, pv, q_rs, kv_rs, _p(dm), *strides, _p(dout), b, s, t, h, kvh, d,
                                0.0, causal))
    torch.cuda.synchronize()
    _close(dout.cpu().numpy(), want, 2e-5, "mha out")


def test_mha_rejects_bad_arguments(ctx):
    assert ctx.lib.b2m_mha_dev(ctx.handle, None, None, None, 64, 64, None, 0, 0, 0, None, 1, 4, 3, 2, 2, 32, 0.0,
                               1) == N.B2M_ERR_INVALID_ARGUMENT     # causal with s > t
    assert ctx.lib.b2m_mha_dev(ctx.handle, None, None, None, 16, 64, None, 0, 0, 0, None, 1, 4, 4, 2, 2, 32, 0.0,
                               0) == N.B2M_ERR_INVALID_ARGUMENT     # q row stride below h * head_dim


@pytest.mark.parametrize("mode", ["precise", "exact"])
def test_tiny_decoder_chain_prefill_and_graph_decode(ctx, mode):
    """Two-layer decoder: prefill, then decode steps replayed as one CUDA
    graph, against the strict composition (oracle MatMulNBits per op).
    PRECISE is held to the path's 1e-3 / 0.99999 contract; EXACT (the
    reference's MatMulNBits order, fp32 attention) to 1e-5. FAST at full depth
    is covered in test_gpu_chains.py."""
    from onnx_runtime_dart_b200.decoder import DecoderConfig, Int4Decoder

    cfg = DecoderConfig.tiny()
    b, s, steps = 2, 6, 3
    md = N.MODE_PRECISE if mode == "precise" else N.MODE_EXACT
    tol, min_cos = (1e-3, 0.99999) if mode == "precise" else (1e-5, 0.9999999)
    dec = Int4Decoder(ctx, cfg, batch=b, cap=s + steps + 1, max_prefill=s, seed=21, keep_host=True, mode=md)
    rng = np.random.default_rng(22)
    prompt = rng.integers(0, cfg.vocab, (b, s)).astype(np.int64)
    dec.prefill(prompt)
    torch.cuda.synchronize()
    want, past = chain_refs.ref_decoder(dec, prompt, None)
    assert_fast_close(dec.logits.cpu().numpy(), want, "prefill logits", max_rel=tol, min_cos=min_cos)
    toks = dec.next_ids.cpu().numpy()
    gen = dec.decode(steps).cpu().numpy()
    cur = toks
    for i in range(steps):
        want, past = chain_refs.ref_decoder(dec, cur.reshape(b, 1), past)
        # the GPU's logits after the last replay correspond to step steps-1
        if i == steps - 1:
            assert_fast_close(dec.logits.cpu().numpy(), want, "decode logits", max_rel=tol, min_cos=min_cos)
        cur = gen[i]
    assert gen.shape == (steps, b)
    assert np.all((gen >= 0) & (gen < cfg.vocab))


@pytest.mark.parametrize("mode,heads", [("fast", 4), ("exact", 4), ("fast", 2)])
def test_tiny_bert_chain_matches_composition(ctx, mode, heads):
    # heads=2 gives head_dim 64: the tensor-core attention kernel.
    from onnx_runtime_dart_b200.bert import BertConfig, BertEncoder

    cfg = BertConfig.tiny()
    cfg.heads = heads
    b, s = 3, 40
    enc = BertEncoder(ctx, cfg, b, s, seed=5, mode=N.MODE_FAST if mode == "fast" else N.MODE_EXACT, keep_host=True)
    rng = np.random.default_rng(9)
    ids = rng.integers(0, cfg.vocab, (b, s), dtype=np.int64)
    mask01 = np.ones((b, s), np.int64)
    mask01[1, 31:] = 0
    want = chain_refs.ref_bert(enc, ids, mask01)
    eager = enc.forward(ids, mask01, use_graph=False)
    graph = enc.forward(ids, mask01, use_graph=True)
    np.testing.assert_array_equal(graph, eager)
    got = graph.astype(np.float64)
    err = float(np.max(np.abs(got - want))) / float(np.max(np.abs(want)))
    cos = float((got * want).sum() / np.sqrt((got * got).sum() * (want.astype(np.float64) ** 2).sum()))
    # Tolerance: each Gemm of the FAST chain is within 1e-3 of the exact one;
    # attention / LayerNorm / GELU add float32 rounding-order differences.
    assert err <= (1e-3 if mode == "fast" else 1e-4), f"bert chain max rel err {err:.3e}"
    assert cos >= 0.99999, f"bert chain cosine {cos:.7f}"


class _DeviceGlue:
    """The device ops behind the fixture runner's interface (tests/glue_fixtures.py)."""

    def __init__(self, ctx):
        self.ctx, self.lib, self.h = ctx, ctx.lib, ctx.handle

    def _run(self):
        torch.cuda.synchronize()

    def gelu(self, x):
        dx = _d(x)
        dy = torch.empty_like(dx)
        N.check(self.lib.b2m_gelu_dev(self.h, _p(dx), _p(dy), dx.numel()))
        self._run()
        return dy.cpu().numpy()

    def rmsnorm(self, x, gamma, eps, skip):
        d = x.shape[-1]
        dx, dg = _d(x), _d(np.asarray(gamma, np.float32))
        ds = _d(skip) if skip is not None else None
        dy, dsum = torch.empty_like(dx), torch.empty_like(dx)
        N.check(self.lib.b2m_rmsnorm_dev(self.h, _p(dx), _p(ds), _p(dg), _p(dy), _p(dsum), dx.numel() // d, d,
                                         ctypes.c_double(eps)))
        self._run()
        return dy.cpu().numpy(), (dsum.cpu().numpy() if skip is not None else None)

    def argmax_last(self, x):
        x = np.ascontiguousarray(x)
        v = x.shape[-1]
        dx = _d(x)
        dout = torch.empty(x.size // v, dtype=torch.int64, device="cuda")
        N.check(self.lib.b2m_argmax_dev(self.h, _p(dx), _p(dout), x.size // v, v))
        self._run()
        return dout.cpu().numpy().reshape(x.shape[:-1])

    def rotary(self, x, pos, cos, sin, heads, interleaved):
        b, s, hid = x.shape
        dx, dp = _d(x), _d(np.asarray(pos, np.int64))
        dc, dsn = _d(cos), _d(sin)
        dy = torch.empty_like(dx)
        half = cos.shape[-1]
        hd = hid // heads
        N.check(self.lib.b2m_rotary_dev(self.h, _p(dx), hid, _p(dp), int(np.asarray(pos).ndim == 2), _p(dc),
                                        _p(dsn), half, cos.shape[0], _p(dy), hid, b, s, heads, hd, min(2 * half, hd),
                                        int(interleaved)))
        self._run()
        return dy.cpu().numpy()

    def gqa(self, q, k, v, h, kvh, pk, pv, cos, sin, scale):
        b, s, _ = q.shape
        d = q.shape[-1] // h
        past = 0 if pk is None else pk.shape[2]
        cap = past + s
        kc = np.zeros((b, kvh, cap, d), np.float32)
        vc = np.zeros((b, kvh, cap, d), np.float32)
        if past:
            kc[:, :, :past], vc[:, :, :past] = pk, pv
        dq, dk, dv, dkc, dvc = _d(q), _d(k), _d(v), _d(kc), _d(vc)
        dpast = _d(np.full(b, past, np.int32))
        dc, dsn = (_d(cos), _d(sin)) if cos is not None else (None, None)
        dout = torch.empty_like(dq)
        half = cos.shape[-1] if cos is not None else 0
        N.check(self.lib.b2m_gqa_dev(self.h, _p(dq), _p(dk), _p(dv), h * d, kvh * d, _p(dkc), _p(dvc), _p(dpast),
                                     _p(dc), _p(dsn), half, 2 * half if cos is not None else 0, 0, _p(dout), b, s, h,
                                     kvh, d, cap, ctypes.c_float(scale)))
        self._run()
        return dout.cpu().numpy(), dkc.cpu().numpy(), dvc.cpu().numpy()

    def mha(self, q, k, v, h, bias, scale):
        b, s, hid = q.shape
        t = k.shape[1]
        d = hid // h
        dq, dk, dv = _d(q), _d(k), _d(v)
        dm, strides = None, (0, 0, 0)
        if bias is not None:
            bh = bias.shape[1]
            dm, strides = _d(bias), (bh * s * t, s * t if bh > 1 else 0, t)
        dout = torch.empty_like(dq)
        N.check(self.lib.b2m_mha_dev(self.h, _p(dq), _p(dk), _p(dv), hid, hid, _p(dm), *strides, _p(dout), b, s, t, h,
                                     h, d, ctypes.c_float(scale), 0))
        self._run()
        return dout.cpu().numpy()


@pytest.mark.parametrize("case", GLUE_CASES)
def test_glue_device_matches_reference_fixture(ctx, case):
    g = load_golden(case)
    got = run_case(g, _DeviceGlue(ctx))
    for name, arr in got.items():
        want = g["expected_arrays"][name]
        if want.dtype.kind in "iu":
            assert np.asarray(arr).astype(np.int64).tolist() == want.tolist(), f"{case}:{name}"
        else:
            assert_fixture_close(arr, want, f"{case}:{name}")


@pytest.mark.parametrize("rows,v", [(64, 151936), (3, 1000), (1, 7), (130, 4099)])
def test_argmax_chunked_ties_nan(ctx, rows, v):
    # Two-pass argmax over row chunks: the smallest index among equal maxima
    # wins across chunk boundaries, NaN never wins, an all -inf row gives 0.
    rng = np.random.default_rng(rows + v)
    x = rng.standard_normal((rows, v)).astype(np.float32)
    x[0, [v // 3, v - 1, 5 % v]] = 50.0                     # ties in different chunks
    if rows > 1:
        x[1] = -np.inf
    if rows > 2:
        x[2, ::3] = np.nan
    dx = _d(x)
    dout = torch.empty(rows, dtype=torch.int64, device="cuda")
    N.check(ctx.lib.b2m_argmax_dev(ctx.handle, _p(dx), _p(dout), rows, v))
    torch.cuda.synchronize()
    vals = np.where(np.isnan(x), -np.inf, x)
    mx = vals.max(axis=1)
    want = np.where(mx >= -np.finfo(np.float32).max, np.argmax(vals == mx[:, None], axis=1), 0)
    np.testing.assert_array_equal(dout.cpu().numpy(), want)
