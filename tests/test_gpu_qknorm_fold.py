"""GPU tests of b2m_gqa_qknorm_dev: the q / k head RMSNorm folded into the
GroupQueryAttention call.

A Qwen3 layer normalises every query and key head (the q_norm / k_norm
SimplifiedLayerNormalization nodes, lib/src/onnx_ops.dart:1771) between the
q/k/v projection and GroupQueryAttention (:1844). The reference runs them as
separate kernels; here a single-token call normalises inside the decode
attention kernel, which also rotates and appends the token's key and value,
and a multi-token call normalises in place before the append. Every case is
held to bit equality with the unfolded sequence (b2m_rmsnorm_head_rows_dev,
then b2m_gqa_dev / b2m_gqa_f16_dev): output, f16 copy and both caches."""
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


def _vp(addr):
    return ctypes.c_void_p(addr)


@pytest.fixture(scope="module")
def ctx():
    c = b2m.Context(0)
    yield c
    c.close()


def _rope(cap, D):
    half = D // 2
    inv = 1.0 / (1000000.0 ** (np.arange(half) * 2.0 / D))
    ang = np.arange(cap)[:, None] * inv[None, :]
    return (torch.from_numpy(np.cos(ang).astype(np.float32)).cuda(),
            torch.from_numpy(np.sin(ang).astype(np.float32)).cuda())


def _run_pair(ctx, rng, b, s, H, KVH, D, cap, pasts, packed, f16):
    """Runs the unfolded and the folded sequence on the same inputs; returns
    both results (out, out16, k cache, v cache)."""
    lib, h = ctx.lib, ctx.handle
    eps = 1e-6
    T = b * s
    gain = torch.from_numpy((1 + 0.2 * rng.standard_normal((H + KVH, D))).astype(np.float32)).cuda()
    cache0 = torch.from_numpy(rng.standard_normal((b, KVH, cap, D)).astype(np.float32)).cuda()
    cos, sin = _rope(cap, D)
    if packed:  # the fused projection's rows: q heads, k heads, v heads
        rs = (H + 2 * KVH) * D
        rows0 = torch.from_numpy((3 * rng.standard_normal((T, rs))).astype(np.float32)).cuda()
    else:
        q0 = torch.from_numpy((3 * rng.standard_normal((T, H * D))).astype(np.float32)).cuda()
        k0 = torch.from_numpy((3 * rng.standard_normal((T, KVH * D))).astype(np.float32)).cuda()
        v0 = torch.from_numpy(rng.standard_normal((T, KVH * D)).astype(np.float32)).cuda()
    res = []
    for fold in (False, True):
        if packed:
            rows = rows0.clone()
            base = rows.data_ptr()
            qp, kp, vp = base, base + H * D * 4, base + (H + KVH) * D * 4
            q_rs = kv_rs = rs
        else:
            q, k, v = q0.clone(), k0.clone(), v0.clone()
            qp, kp, vp = q.data_ptr(), k.data_ptr(), v.data_ptr()
            q_rs, kv_rs = H * D, KVH * D
        kc, vc = cache0.clone(), cache0.clone()
        past = torch.tensor(pasts, dtype=torch.int32, device="cuda")
        out = torch.full((T, H * D), float("nan"), device="cuda")
        out16 = torch.zeros((T, H * D), device="cuda", dtype=torch.float16)
        torch.cuda.synchronize()
        if fold:
            N.check(lib.b2m_gqa_qknorm_dev(h, _vp(qp), _vp(kp), _vp(vp), q_rs, kv_rs, _p(gain), eps, _p(kc), _p(vc),
                                           _p(past), _p(cos), _p(sin), D // 2, D, 0, _p(out),
                                           _p(out16) if f16 else None, b, s, H, KVH, D, cap, ctypes.c_float(0.0)))
        else:
            if packed:
                N.check(lib.b2m_rmsnorm_head_rows_dev(h, _vp(qp), _p(gain), _vp(qp), T, H + KVH, D, q_rs, eps))
            else:
                N.check(lib.b2m_rmsnorm_head_rows_dev(h, _vp(qp), _p(gain), _vp(qp), T, H, D, q_rs, eps))
                N.check(lib.b2m_rmsnorm_head_rows_dev(h, _vp(kp), _vp(gain.data_ptr() + H * D * 4), _vp(kp), T, KVH,
                                                      D, kv_rs, eps))
            args = [h, _vp(qp), _vp(kp), _vp(vp), q_rs, kv_rs, _p(kc), _p(vc), _p(past), _p(cos), _p(sin), D // 2, D,
                    0, _p(out)]
            tail = [b, s, H, KVH, D, cap, ctypes.c_float(0.0)]
            if f16:
                N.check(lib.b2m_gqa_f16_dev(*args, _p(out16), *tail))
            else:
                N.check(lib.b2m_gqa_dev(*args, *tail))
        N.check(lib.b2m_synchronize(h))
        res.append((out, out16, kc, vc))
    return res


@pytest.mark.parametrize("b,pasts_kind,H,KVH,D,packed,f16", [
    (64, "ragged", 16, 8, 128, True, True),    # the config-5 decode step
    (64, "ragged", 16, 8, 128, True, False),
    (3, "edges", 16, 8, 128, False, True),     # separate q / k buffers
    (8, "ragged", 8, 8, 64, True, True),       # one query head per kv head
    (5, "edges", 32, 4, 64, False, False),     # eight query heads per kv head
    (4, "ragged", 12, 4, 96, True, True),
])
def test_decode_fold_same_bits(ctx, b, pasts_kind, H, KVH, D, packed, f16):
    """One token per sequence: the decode kernel's own norm, rotary and
    append against the separate launches, with key splits (ragged positions
    from 0 to the last free slot)."""
    rng = np.random.default_rng(b * 7 + D)
    cap = 600
    if pasts_kind == "ragged":
        pasts = rng.integers(0, cap, b).tolist()
    else:
        pasts = ([0, cap - 1, 1, 129, 257] * b)[:b]
    ref, got = _run_pair(ctx, rng, b, 1, H, KVH, D, cap, pasts, packed, f16)
    for r, g in zip(ref, got):
        assert torch.equal(r, g)
    if f16:
        assert torch.equal(got[1], got[0].half())


@pytest.mark.parametrize("b,s,D,packed", [(4, 40, 128, True), (2, 17, 128, False), (3, 150, 64, True),
                                          (2, 9, 96, True)])
def test_prefill_fold_same_bits(ctx, b, s, D, packed):
    """Several tokens per sequence: the append kernel normalising k and the
    flash kernel normalising q (head_dim 64 / 128; 150 queries span two
    query tiles), and at head_dim 96 the in-place norm before the CUDA-core
    kernel, against the separate launches."""
    rng = np.random.default_rng(s)
    pasts = [0, 7, 3, 20][:b]
    ref, got = _run_pair(ctx, rng, b, s, 16, 8, D, 256, pasts, packed, True)
    for r, g in zip(ref, got):
        assert torch.equal(r, g)


@pytest.mark.parametrize("b,s,D", [(64, 1, 128), (3, 1, 128), (4, 40, 128), (2, 9, 96)])
def test_fold_f16_only_output(ctx, b, s, D):
    """out = NULL with out16 given: the f16 output and the caches are the
    same bits as with the fp32 output requested (the decode kernel with and
    without key splits and the flash prefill skip the fp32 rows; at head_dim
    96 the CUDA-core kernel writes them to scratch first)."""
    rng = np.random.default_rng(b * 100 + s)
    lib, h = ctx.lib, ctx.handle
    H, KVH, cap = 16, 8, 256
    T = b * s
    rs = (H + 2 * KVH) * D
    rows0 = torch.from_numpy((3 * rng.standard_normal((T, rs))).astype(np.float32)).cuda()
    gain = torch.from_numpy((1 + 0.2 * rng.standard_normal((H + KVH, D))).astype(np.float32)).cuda()
    cache0 = torch.from_numpy(rng.standard_normal((b, KVH, cap, D)).astype(np.float32)).cuda()
    cos, sin = _rope(cap, D)
    pasts = rng.integers(0, cap - s, b).tolist()
    res = []
    for with_out in (True, False):
        rows = rows0.clone()
        base = rows.data_ptr()
        kc, vc = cache0.clone(), cache0.clone()
        past = torch.tensor(pasts, dtype=torch.int32, device="cuda")
        out = torch.empty((T, H * D), device="cuda")
        out16 = torch.zeros((T, H * D), device="cuda", dtype=torch.float16)
        torch.cuda.synchronize()
        N.check(lib.b2m_gqa_qknorm_dev(h, _vp(base), _vp(base + H * D * 4), _vp(base + (H + KVH) * D * 4), rs, rs,
                                       _p(gain), 1e-6, _p(kc), _p(vc), _p(past), _p(cos), _p(sin), D // 2, D, 0,
                                       _p(out) if with_out else None, _p(out16), b, s, H, KVH, D, cap,
                                       ctypes.c_float(0.0)))
        N.check(lib.b2m_synchronize(h))
        res.append((out16, kc, vc))
    for r, g in zip(res[0], res[1]):
        assert torch.equal(r, g)


def test_decode_fold_cache_full(ctx):
    """A sequence whose cache is full reports the capacity error, as the
    separate append kernel does, and leaves the cache alone."""
    rng = np.random.default_rng(5)
    lib, h = ctx.lib, ctx.handle
    b, H, KVH, D, cap = 2, 16, 8, 128, 64
    qkv = torch.from_numpy(rng.standard_normal((b, (H + 2 * KVH) * D)).astype(np.float32)).cuda()
    gain = torch.ones((H + KVH, D), device="cuda")
    kc = torch.from_numpy(rng.standard_normal((b, KVH, cap, D)).astype(np.float32)).cuda()
    vc = kc.clone()
    k_before = kc.clone()
    cos, sin = _rope(cap, D)
    past = torch.tensor([cap, 3], dtype=torch.int32, device="cuda")
    out = torch.empty((b, H * D), device="cuda")
    base, rs = qkv.data_ptr(), (H + 2 * KVH) * D
    torch.cuda.synchronize()
    with pytest.raises(N.ArgumentError, match="capacity"):
        N.check(lib.b2m_gqa_qknorm_dev(h, _vp(base), _vp(base + H * D * 4), _vp(base + (H + KVH) * D * 4), rs, rs,
                                       _p(gain), 1e-6, _p(kc), _p(vc), _p(past), _p(cos), _p(sin), D // 2, D, 0,
                                       _p(out), None, b, 1, H, KVH, D, cap, ctypes.c_float(0.0)))
        N.check(lib.b2m_synchronize(h))
    assert torch.equal(kc[0], k_before[0])  # the full sequence: nothing appended
    assert not torch.equal(kc[1, :, 3], k_before[1, :, 3])  # the other one appended at 3
    N.check(lib.b2m_synchronize(h))  # the error was reported once and cleared


def test_qknorm_rejects_null_gain(ctx):
    lib, h = ctx.lib, ctx.handle
    with pytest.raises(N.ArgumentError, match="qk_gain"):
        N.check(lib.b2m_gqa_qknorm_dev(h, None, None, None, 0, 0, None, 1e-6, None, None, None, None, None, 0, 0, 0,
                                       None, None, 1, 1, 16, 8, 128, 64, ctypes.c_float(0.0)))


def test_decoder_fold_same_tokens(ctx):
    """Qwen3-0.6B shapes, two layers, 64 sequences: prefill and three decode
    steps (one CUDA graph) with the folded and the separate head norms give
    identical logits and caches."""
    cfg = DecoderConfig.qwen3_0_6b()
    cfg.layers = 2
    B, S = 64, 24
    prompt = np.random.default_rng(9).integers(0, cfg.vocab, (B, S))
    out = []
    for fold in (False, True):
        dec = Int4Decoder(ctx, cfg, batch=B, cap=S + 8, max_prefill=S, seed=13, fold_qk_norm=fold)
        dec.prefill(prompt)
        torch.cuda.synchronize()
        logits = [dec.logits.cpu().numpy().copy()]
        toks = dec.decode(3)
        torch.cuda.synchronize()
        logits.append(dec.logits.cpu().numpy().copy())
        out.append((logits, toks.cpu().numpy(), dec.kcache.cpu().numpy(), dec.vcache.cpu().numpy()))
        del dec
    for a, b_ in zip(out[0][0], out[1][0]):
        np.testing.assert_array_equal(a, b_)
    np.testing.assert_array_equal(out[0][1], out[1][1])
    np.testing.assert_array_equal(out[0][2], out[1][2])
    np.testing.assert_array_equal(out[0][3], out[1][3])
