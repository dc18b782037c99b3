"""CPU-only checks of the C ABI library and the host-side operator layer.

No compute runs here: the library must load without a GPU, export every
entry point include/b2m.h declares, report "no device" cleanly, and the
Python mirror of the reference's operator validation must raise the same
error classes as the reference (onnx_qlinear_ops.dart:126-166) before any
device work.
"""
import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    txt = open(os.path.join(ROOT, "include", "b2m.h")).read()
    return sorted(set(re.findall(r"B2M_API\s+[^;(]*?\b(b2m_\w+)\s*\(", txt)))


@pytest.fixture(scope="module")
def lib():
    from onnx_runtime_dart_b200 import _native, build

    if not os.path.exists(build.LIB):
        build.build()
    return _native.load()


def test_header_symbols_all_exported(lib):
    syms = header_symbols()
    assert len(syms) >= 25
    for s in syms:
        assert hasattr(lib, s), f"libb200mm.so does not export {s}"


def test_python_binding_covers_header(lib):
    from onnx_runtime_dart_b200 import _native

    assert sorted(_native.SIGNATURES) == header_symbols()


def test_abi_version_and_no_device(lib):
    from onnx_runtime_dart_b200 import _native

    assert lib.b2m_abi_version() == 1
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    n = ctypes.c_int32(-1)
    assert lib.b2m_device_count(ctypes.byref(n)) == 0
    assert n.value == 0
    h = ctypes.c_void_p()
    st = lib.b2m_init(0, ctypes.byref(h))
    assert st == _native.B2M_ERR_NO_DEVICE
    assert b"no CUDA device" in lib.b2m_last_error()
    with pytest.raises(_native.NoDeviceError):
        _native.check(st)


def test_null_arguments_are_rejected_not_crashing(lib):
    from onnx_runtime_dart_b200 import _native

    assert lib.b2m_matmul_f32(None, None, None, None, 0, None) == _native.B2M_ERR_INVALID_ARGUMENT
    assert lib.b2m_tensor_free(None) == 0
    assert lib.b2m_weight_free(None) == 0
    assert lib.b2m_shutdown(None) == 0
    assert lib.b2m_tensor_info(None, None, None, None, None) == _native.B2M_ERR_INVALID_ARGUMENT


def test_nbits_prepack_validation_order(lib):
    # bits check first (UnsupportedError), then K/N/block (ArgumentError) —
    # the reference's order (onnx_qlinear_ops.dart:126-136). Context is NULL:
    # the library rejects it before any device call.
    from onnx_runtime_dart_b200 import _native

    assert lib.b2m_weight_prepack_nbits(None, None, None, None, 0, 64, 8, 4, 32, None) == \
        _native.B2M_ERR_INVALID_ARGUMENT


def _nbits_args(k=64, n=8, block=32):
    nb = (k + block - 1) // block
    return (np.zeros((n, nb, block // 2), np.uint8), np.ones((n, nb), np.float32),
            np.zeros((n, (nb + 1) // 2), np.uint8))


def test_validate_nbits_mirrors_reference():
    from onnx_runtime_dart_b200 import ArgumentError, UnsupportedError, validate_nbits

    bq, sc, zp = _nbits_args()
    validate_nbits([2, 64], np.float32, bq, sc, zp, None, 64, 8, 4, 32)
    with pytest.raises(UnsupportedError, match="only bits=4"):
        validate_nbits([2, 64], np.float32, bq, sc, zp, None, 64, 8, 8, 32)
    for k, n, blk, shape in [(0, 8, 32, [2, 0]), (64, 0, 32, [2, 64]), (64, 8, 8, [2, 64]),
                             (64, 8, 48, [2, 64]), (64, 8, 32, [2, 63]), (64, 8, 32, [])]:
        with pytest.raises(ArgumentError, match="invalid K, N, block_size or input shape"):
            validate_nbits(shape, np.float32, bq, sc, zp, None, k, n, 4, blk)
    with pytest.raises(ArgumentError, match="invalid packed weights or scales"):
        validate_nbits([2, 64], np.float32, bq.astype(np.int8), sc, zp, None, 64, 8, 4, 32)
    with pytest.raises(ArgumentError, match="invalid packed weights or scales"):
        validate_nbits([2, 64], np.int32, bq, sc, zp, None, 64, 8, 4, 32)
    with pytest.raises(ArgumentError, match="invalid packed weights or scales"):
        validate_nbits([2, 64], np.float32, bq, sc.reshape(2, 8), zp, None, 64, 8, 4, 32)
    with pytest.raises(ArgumentError, match="invalid zero_points"):
        validate_nbits([2, 64], np.float32, bq, sc, zp[:5], None, 64, 8, 4, 32)
    with pytest.raises(ArgumentError, match="invalid zero_points"):
        validate_nbits([2, 64], np.float32, bq, sc, np.zeros((8, 1), np.int32), None, 64, 8, 4, 32)
    validate_nbits([2, 64], np.float32, bq, sc, np.zeros((8, 2), np.float32), None, 64, 8, 4, 32)
    with pytest.raises(ArgumentError, match="bias must be floating point"):
        validate_nbits([2, 64], np.float32, bq, sc, zp, np.zeros(8, np.int32), 64, 8, 4, 32)
    with pytest.raises(ArgumentError, match="bias must be floating point"):
        validate_nbits([2, 64], np.float32, bq, sc, zp, np.zeros((1, 8), np.float32), 64, 8, 4, 32)


def test_dispatch_rejects_g_idx_before_device_work():
    from onnx_runtime_dart_b200 import UnsupportedError
    from onnx_runtime_dart_b200.dispatch import GpuDispatch

    bq, sc, zp = _nbits_args()
    d = GpuDispatch(ctx=None, initializers={"B": bq})
    with pytest.raises(UnsupportedError, match="g_idx"):
        d.dispatch("MatMulNBits", ["A", "B", "S", "", "G"], [np.zeros((1, 64), np.float32), bq, sc, None, None],
                   {"K": 64, "N": 8, "block_size": 32})
    assert d.dispatch("Relu", ["x"], [np.zeros(2)], {}) is None


def test_product_path_has_no_oracle_or_cpu_fallback():
    # The product package must not import the oracle (test infrastructure).
    pkg = os.path.join(ROOT, "onnx_runtime_dart_b200")
    for f in os.listdir(pkg):
        if f.endswith(".py"):
            src = open(os.path.join(pkg, f)).read()
            assert not re.search(r"^\s*(import|from)\s+oracle\b", src, re.M), f


def test_conv_spatial_attributes_are_length_checked():
    # The C ABI reads kernel_shape[nd], strides[nd], pads[2 nd], dilations[nd];
    # the Python layer rejects arrays of other lengths before any call.
    from types import SimpleNamespace

    from onnx_runtime_dart_b200 import _native as N
    from onnx_runtime_dart_b200 import ops

    pw = SimpleNamespace(shape=(8, 4, 3, 3))
    (ks, _), (st, _), (pd, _), (dl, _) = ops._spatial_attrs(pw, [1, 2], [1, 1, 0, 0], None)
    assert ks.tolist() == [3, 3] and st.tolist() == [1, 2] and pd.tolist() == [1, 1, 0, 0] and dl is None
    with pytest.raises(N.ArgumentError, match="pads"):
        ops._spatial_attrs(pw, None, [1, 1], None)
    with pytest.raises(N.ArgumentError, match="strides"):
        ops._spatial_attrs(pw, [1], None, None)
    with pytest.raises(N.ArgumentError, match="dilations"):
        ops._spatial_attrs(pw, None, None, [1, 1, 1])
    with pytest.raises(N.ArgumentError, match="rank"):
        ops._check_conv_rank(np.zeros((1, 4, 5)), pw, 3, 5)
    assert ops.AUTO_PAD == {"NOTSET": 0, "SAME_UPPER": 1, "SAME_LOWER": 2, "VALID": 3}


def test_swiglu_row_order_is_the_tile_interleave():
    """The gate / up row order b2m_matmul_nbits_swiglu_dev takes: per 128-row
    tile t, gate rows 64t .. 64t+63, then the matching up rows."""
    from onnx_runtime_dart_b200.decoder import swiglu_row_order

    inter = 3072
    r = swiglu_row_order(inter)
    assert sorted(r.tolist()) == list(range(2 * inter))
    t = r.reshape(inter // 64, 2, 64)
    base = np.arange(inter // 64)[:, None] * 64 + np.arange(64)[None, :]
    np.testing.assert_array_equal(t[:, 0, :], base)
    np.testing.assert_array_equal(t[:, 1, :], base + inter)


def test_fused_entries_reject_bad_arguments_without_a_device(lib):
    """The fused attention and SwiGLU entries validate before touching a
    device: a null context, a null gain table, a negative epsilon."""
    from onnx_runtime_dart_b200 import _native

    bad = _native.B2M_ERR_INVALID_ARGUMENT
    assert lib.b2m_matmul_nbits_swiglu_dev(None, None, None, 4, None, 1, None, None) == bad

    def qknorm(gain, eps, b, s):  # a null context and null buffers; h 16, kvh 8, head_dim 128, cap 64
        return lib.b2m_gqa_qknorm_dev(None, None, None, None, 0, 0, gain, eps, None, None, None, None, None, 0, 0, 0,
                                      None, None, b, s, 16, 8, 128, 64, ctypes.c_float(0.0))
    assert qknorm(None, 1e-6, 1, 1) == bad
    assert b"qk_gain" in lib.b2m_last_error()
    g = np.ones((24, 128), np.float32)
    assert qknorm(g.ctypes.data_as(ctypes.c_void_p), -1.0, 1, 1) == bad
    assert b"eps" in lib.b2m_last_error()
    assert qknorm(None, 1e-6, 0, 0) == bad  # nothing to do, but the context is still checked
