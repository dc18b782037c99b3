"""GPU tests of b2m_matmul_nbits_swiglu_dev: a layer's gate / up MatMulNBits
and the SiLU*Mul between them and the down projection in one call.

The reference runs the gate and up MatMulNBits (opMatMulNBits,
lib/src/onnx_qlinear_ops.dart:115-228) and then the Sigmoid / Mul / Mul
nodes as separate kernels. The fused weight's rows are tile-interleaved (64
gate rows, then the 64 matching up rows, per 128-row tile) so that on the
tensor-core route each CTA of the GEMM forms silu(gate) * up in its epilogue
and no fp32 gate / up rows reach memory; other routes run the GEMM and one
elementwise pass. Every case is held to bit equality with the separate calls
on the same weight (b2m_matmul_nbits_dev, the gate / up columns gathered, then
b2m_silu_mul_f16_dev), across the routes: the decode GEMV (1 and 8 rows), the
tensor-core kernel with K split over a cluster (33 and 64 rows of a
3072-column weight) and unsplit (64 to 2048 rows of 6144 columns), PRECISE
and EXACT; and a decoder with the fused call against one without, on
its tolerance contract."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
import onnx_runtime_dart_b200 as b2m  # noqa: E402
from onnx_runtime_dart_b200 import _native as N  # noqa: E402
from onnx_runtime_dart_b200.decoder import DecoderConfig, Int4Decoder, swiglu_row_order  # noqa: E402


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.fixture(scope="module")
def ctx():
    c = b2m.Context(0)
    yield c
    c.close()


def _interleaved_weight(ctx, rng, k, inter):
    nb = k // 32
    n = 2 * inter
    bq = rng.integers(0, 256, (n, nb, 16), dtype=np.uint8)
    sc = (np.abs(rng.normal(0, 0.02, (n, nb))) + 1e-3).astype(np.float32)
    zp = rng.integers(0, 256, (n, (nb + 1) // 2), dtype=np.uint8)
    r = swiglu_row_order(inter)
    return ctx.prepack_nbits(bq[r], sc[r], zp[r], k, n, 4, 32)


def _separate(ctx, a, w, m, inter, mode):
    """b2m_matmul_nbits_dev on the interleaved weight, the gate / up columns
    gathered, then b2m_silu_mul_f16_dev: (act, act16)."""
    lib, h = ctx.lib, ctx.handle
    y = torch.empty((m, 2 * inter), device="cuda")
    N.check(lib.b2m_matmul_nbits_dev(h, _p(a), m, w.handle, None, mode, _p(y)))
    N.check(lib.b2m_synchronize(h))  # the library's stream, then torch's
    t = y.view(m, inter // 64, 2, 64)
    gate = t[:, :, 0, :].reshape(m, inter).contiguous()
    up = t[:, :, 1, :].reshape(m, inter).contiguous()
    act = torch.empty((m, inter), device="cuda")
    act16 = torch.empty((m, inter), device="cuda", dtype=torch.float16)
    torch.cuda.synchronize()
    N.check(lib.b2m_silu_mul_f16_dev(h, _p(gate), _p(up), inter, inter, _p(act), _p(act16), m, inter))
    N.check(lib.b2m_synchronize(h))
    return act, act16


def _fused(ctx, a, a16, w, m, inter, mode, want_act=True, want16=True):
    lib, h = ctx.lib, ctx.handle
    act = torch.full((m, inter), float("nan"), device="cuda")
    act16 = torch.zeros((m, inter), device="cuda", dtype=torch.float16)
    a16 = a16.contiguous() if a16 is not None else None
    torch.cuda.synchronize()  # torch's fills before the library's stream reads or writes
    N.check(lib.b2m_matmul_nbits_swiglu_dev(h, _p(a) if a is not None else None, _p(a16) if a16 is not None else None,
                                            m, w.handle, mode, _p(act) if want_act else None,
                                            _p(act16) if want16 else None))
    N.check(lib.b2m_synchronize(h))
    return act, act16


@pytest.mark.parametrize("m,mode,inter", [
    (1, N.MODE_FAST, 3072), (8, N.MODE_FAST, 3072),     # decode GEMV
    (64, N.MODE_FAST, 3072),                              # 48 column tiles: unsplit
    (64, N.MODE_FAST, 1536), (33, N.MODE_FAST, 1536),    # 24 column tiles: K split over a cluster
    (200, N.MODE_FAST, 3072), (2048, N.MODE_FAST, 3072),
    (8, N.MODE_PRECISE, 3072), (96, N.MODE_PRECISE, 3072), (5, N.MODE_EXACT, 3072)])
def test_swiglu_matches_separate_calls_bitwise(ctx, m, mode, inter):
    rng = np.random.default_rng(m * 3 + mode)
    k = 1024
    w = _interleaved_weight(ctx, rng, k, inter)
    a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    torch.cuda.synchronize()
    act_ref, act16_ref = _separate(ctx, a, w, m, inter, mode)
    act, act16 = _fused(ctx, a, None, w, m, inter, mode)
    assert torch.equal(act, act_ref)
    assert torch.equal(act16, act16_ref)
    if mode == N.MODE_FAST:  # the producer-written f16 operand: the same bits again
        act_b, act16_b = _fused(ctx, a, a.half(), w, m, inter, mode)
        assert torch.equal(act_b, act_ref)
        assert torch.equal(act16_b, act16_ref)
    w.free()


@pytest.mark.parametrize("m", [64, 1000])
def test_swiglu_single_outputs(ctx, m):
    """Only act16 (the down projection's f16 operand) or only act."""
    rng = np.random.default_rng(m)
    k, inter = 1024, 1536
    w = _interleaved_weight(ctx, rng, k, inter)
    a = torch.from_numpy(rng.standard_normal((m, k)).astype(np.float32)).cuda()
    torch.cuda.synchronize()
    act_ref, act16_ref = _separate(ctx, a, w, m, inter, N.MODE_FAST)
    act, act16 = _fused(ctx, a, a.half(), w, m, inter, N.MODE_FAST, want_act=False)
    assert torch.equal(act16, act16_ref)
    assert torch.isnan(act).all()  # untouched
    act, act16 = _fused(ctx, a, None, w, m, inter, N.MODE_FAST, want16=False)
    assert torch.equal(act, act_ref)
    assert not act16.any()  # untouched
    w.free()


def test_swiglu_argument_errors(ctx):
    rng = np.random.default_rng(1)
    lib, h = ctx.lib, ctx.handle
    a = torch.zeros((4, 256), device="cuda")
    act = torch.zeros((4, 160), device="cuda")
    w_odd = _interleaved_weight(ctx, rng, 256, 192)  # N = 384 = 3 x 128: accepted
    w_bad = ctx.prepack_nbits(rng.integers(0, 256, (320, 8, 16), dtype=np.uint8),
                              np.ones((320, 8), np.float32), None, 256, 320, 4, 32)  # N % 128 != 0
    with pytest.raises(N.ArgumentError, match="multiple of 128"):
        N.check(lib.b2m_matmul_nbits_swiglu_dev(h, _p(a), None, 4, w_bad.handle, N.MODE_FAST, _p(act), None))
    with pytest.raises(N.ArgumentError, match="bad pointers"):
        N.check(lib.b2m_matmul_nbits_swiglu_dev(h, _p(a), None, 4, w_odd.handle, N.MODE_FAST, None, None))
    with pytest.raises(N.UnsupportedError, match="fp32 activations"):  # the GEMV route needs fp32 rows
        N.check(lib.b2m_matmul_nbits_swiglu_dev(h, None, _p(a.half()), 4, w_odd.handle, N.MODE_FAST, _p(act), None))
    w_odd.free()
    w_bad.free()


def test_decoder_swiglu_within_contract(ctx):
    """Qwen3-0.6B shapes, two layers, 64 sequences, FAST: the decoder with the
    fused gate / up / SiLU*Mul call against the separate calls (stacked
    weight rows, so the GEMM's column tiles, and with them its summation
    order, differ): prefill logits and one decode step from the same tokens
    within the FAST per-op contract."""
    cfg = DecoderConfig.qwen3_0_6b()
    cfg.layers = 2
    B, S = 64, 32
    prompt = np.random.default_rng(21).integers(0, cfg.vocab, (B, S))
    decs, logits = [], []
    for sw in (False, True):
        dec = Int4Decoder(ctx, cfg, batch=B, cap=S + 4, max_prefill=S, seed=17, swiglu_epilogue=sw)
        assert dec.swiglu == sw
        dec.prefill(prompt)
        torch.cuda.synchronize()
        logits.append(dec.logits.cpu().numpy().copy())
        decs.append(dec)
    decs[1].next_ids.copy_(decs[0].next_ids)
    torch.cuda.synchronize()
    for d in decs:
        d.decode(1, use_graph=False)
    torch.cuda.synchronize()
    step = [d.logits.cpu().numpy().copy() for d in decs]
    for have, want in ((logits[1], logits[0]), (step[1], step[0])):
        h64, w64 = have.astype(np.float64).ravel(), want.astype(np.float64).ravel()
        rel = np.max(np.abs(h64 - w64)) / np.max(np.abs(w64))
        cos = np.dot(h64, w64) / np.sqrt(np.dot(h64, h64) * np.dot(w64, w64))
        assert rel <= 1e-3 and cos >= 0.99999, (rel, cos)
