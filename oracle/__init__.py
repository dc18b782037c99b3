"""CPU oracle for the MatMul-family hot path — TEST INFRASTRUCTURE ONLY.

A numpy/ctypes front end for ``b2m_oracle.c``, the C restatement of the
reference Dart arithmetic (``lib/src/gemm_kernel_simd.dart``,
``lib/src/onnx_ops.dart:1710-1766, 2152-2173``,
``lib/src/onnx_qlinear_ops.dart:19-228``). Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference arm may
import this package; the product library never links or calls it.

Pinning: the C restatement is checked against the ORT-generated golden vectors
the reference's own fixture-parity test replays (``tests/golden/``, made by
``tests/golden/make_golden.py`` from ``test/fixtures/*``), with the reference's
tolerances (``test/fixture_parity_test.dart:21, 65-108``): integer outputs
exact, float outputs max|d| <= max(2e-5, 2e-5*max|ref|) and cosine > 0.999999.
The Dart VM itself cannot run here (no Dart SDK), so bitwise identity with the
Dart VM rests on the restated rounding rules, not on a Dart run.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i64 = ctypes.c_int64


def build() -> str:
    """Compile the oracle with its Makefile (gcc, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
        os.path.join(_HERE, "b2m_oracle.c")
    ):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    lib.orc_matmul_kernel.argtypes = [_f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, ctypes.c_int]
    lib.orc_matmul_kernel.restype = None
    lib.orc_matmul.argtypes = [_f32p, _i64p, ctypes.c_int, _f32p, _i64p, ctypes.c_int, _f32p, ctypes.c_int]
    lib.orc_matmul.restype = ctypes.c_int
    lib.orc_gemm.argtypes = [_f32p, _i64, _i64, _f32p, _i64, _i64, _f32p, _i64p, ctypes.c_int,
                             ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_int, _f32p, ctypes.c_int]
    lib.orc_gemm.restype = ctypes.c_int
    mmi = [_i32p, _i64, _i64, _i64, _i32p, _i64, _i64, _i32p, _i64, _i32p, _i64]
    lib.orc_matmul_integer.argtypes = mmi + [_i64p, ctypes.c_int]
    lib.orc_matmul_integer.restype = ctypes.c_int
    lib.orc_qlinear_matmul.argtypes = mmi + [ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                             ctypes.c_int32, ctypes.c_int32, ctypes.c_int32, _i64p, ctypes.c_int]
    lib.orc_qlinear_matmul.restype = ctypes.c_int
    lib.orc_qlinear_multiplier.argtypes = [ctypes.c_float] * 3
    lib.orc_qlinear_multiplier.restype = ctypes.c_float
    lib.orc_round_even.argtypes = [ctypes.c_double]
    lib.orc_round_even.restype = ctypes.c_int64
    lib.orc_dynamic_quantize_linear.argtypes = [_f32p, _i64, _u8p, ctypes.POINTER(ctypes.c_float)]
    lib.orc_dynamic_quantize_linear.restype = ctypes.c_int64
    lib.orc_matmul_nbits.argtypes = [_f32p, _i64, _i64, _u8p, _f32p, _u8p, _f32p, _f32p, _i64, _i64, _f32p, ctypes.c_int]
    lib.orc_matmul_nbits.restype = ctypes.c_int
    lib.orc_nbits_dequant.argtypes = [_u8p, _f32p, _u8p, _f32p, _i64, _i64, _i64, _f32p]
    lib.orc_nbits_dequant.restype = None
    lib.orc_conv_f32.argtypes = [_f32p, _i64p, ctypes.c_int, _f32p, _i64p, _i64, _f32p, _i64p, _i64p, _i64p, _i64,
                                 _f32p]
    lib.orc_conv_f32.restype = ctypes.c_int
    lib.orc_conv_int_acc.argtypes = [_i32p, _i64, _i64, _i64, _i64, _i32p, _i64, _i64, _i64, _i64, ctypes.c_int32,
                                     _i32p] + [_i64] * 9 + [_i64p]
    lib.orc_conv_int_acc.restype = None
    lib.orc_qlinear_conv_requant.argtypes = [_i64p, _i64, _i64, _i64, ctypes.c_double,
                                             ctypes.POINTER(ctypes.c_double), _i64, ctypes.c_double, _i64, _i64p,
                                             _i64, _i64, _i64p]
    lib.orc_qlinear_conv_requant.restype = None
    lib.orc_conv_transpose_f32.argtypes = [_f32p, _i64p, ctypes.c_int, _f32p, _i64p, _i64, _i64, _f32p, _i64p,
                                           _i64p, _i64p, _i64p, _i64p, _f32p, _i64p]
    lib.orc_conv_transpose_f32.restype = ctypes.c_int
    lib.orc_conv_winograd_f2x2.argtypes = [_f32p, _i64, _i64, _i64, _i64, _f32p, _i64, _f32p, _i64, _f32p]
    lib.orc_conv_winograd_f2x2.restype = ctypes.c_int
    _lib = lib
    return lib


def _p(arr, typ):
    return None if arr is None else arr.ctypes.data_as(typ)


def _c(arr, dtype):
    return None if arr is None else np.ascontiguousarray(arr, dtype=dtype)


def matmul_kernel(a, b, m, k, n, nthreads=1):
    """``matmulKernel`` on fresh zeroed output (gemm_kernel_simd.dart:32)."""
    a = _c(a, np.float32)
    b = _c(b, np.float32)
    out = np.zeros(m * n, np.float32)
    _load().orc_matmul_kernel(_p(a, _f32p), _p(b, _f32p), _p(out, _f32p), m, k, n, n, nthreads)
    return out.reshape(m, n)


def _broadcast(a_batch, b_batch):
    rank = max(len(a_batch), len(b_batch))
    ap = [1] * (rank - len(a_batch)) + list(a_batch)
    bp = [1] * (rank - len(b_batch)) + list(b_batch)
    out = []
    for x, y in zip(ap, bp):
        if x == y or y == 1:
            out.append(x)
        elif x == 1:
            out.append(y)
        else:
            raise ValueError(f"Cannot broadcast shapes {a_batch} and {b_batch}")
    return out


def matmul(a, b, nthreads=1):
    """``opMatMul`` (onnx_ops.dart:1710): numpy-broadcast batched fp32 MatMul."""
    a = _c(a, np.float32)
    b = _c(b, np.float32)
    out_shape = _broadcast(a.shape[:-2], b.shape[:-2]) + [a.shape[-2], b.shape[-1]]
    out = np.zeros(int(np.prod(out_shape)), np.float32)
    ash = np.array(a.shape, np.int64)
    bsh = np.array(b.shape, np.int64)
    rc = _load().orc_matmul(_p(a, _f32p), _p(ash, _i64p), a.ndim, _p(b, _f32p), _p(bsh, _i64p), b.ndim,
                            _p(out, _f32p), nthreads)
    if rc:
        raise ValueError("oracle matmul: bad shapes")
    return out.reshape(out_shape)


def gemm(a, b, c=None, alpha=1.0, beta=1.0, transA=False, transB=False, nthreads=1):
    """``opGemm`` (onnx_ops.dart:2152-2173)."""
    a = _c(a, np.float32)
    b = _c(b, np.float32)
    c = _c(c, np.float32)
    M = a.shape[1] if transA else a.shape[0]
    N = b.shape[0] if transB else b.shape[1]
    y = np.zeros(M * N, np.float32)
    csh = None if c is None else np.array(c.shape, np.int64)
    rc = _load().orc_gemm(_p(a, _f32p), a.shape[0], a.shape[1], _p(b, _f32p), b.shape[0], b.shape[1],
                          _p(c, _f32p), _p(csh, _i64p), 0 if c is None else c.ndim,
                          float(np.float32(alpha)), float(np.float32(beta)), int(bool(transA)),
                          int(bool(transB)), _p(y, _f32p), nthreads)
    if rc:
        raise ValueError("oracle gemm: bad shapes")
    return y.reshape(M, N)


def _int_operands(a, b, a_zp, b_zp):
    a = np.asarray(a)
    b = np.asarray(b)
    m, k = a.shape[-2], a.shape[-1]
    n = b.shape[-1]
    a_batch = a.size // (m * k) if m * k else 1
    b_batch = b.size // (k * n) if k * n else 1
    a32 = _c(a.reshape(-1), np.int32)
    b32 = _c(b.reshape(-1), np.int32)
    az = None if a_zp is None else _c(np.asarray(a_zp).reshape(-1), np.int32)
    bz = None if b_zp is None else _c(np.asarray(b_zp).reshape(-1), np.int32)
    batch_shape = list(a.shape[:-2]) if a_batch >= b_batch else list(b.shape[:-2])
    return a32, b32, az, bz, m, k, n, a_batch, b_batch, batch_shape


def matmul_integer(a, b, a_zp=None, b_zp=None, nthreads=1):
    """``opMatMulInteger`` (onnx_qlinear_ops.dart:32-81); int64 result."""
    a32, b32, az, bz, m, k, n, ab, bb, bs = _int_operands(a, b, a_zp, b_zp)
    out = np.zeros(max(ab, bb) * m * n, np.int64)
    rc = _load().orc_matmul_integer(_p(a32, _i32p), ab, m, k, _p(b32, _i32p), bb, n, _p(az, _i32p),
                                    0 if az is None else az.size, _p(bz, _i32p), 0 if bz is None else bz.size,
                                    _p(out, _i64p), nthreads)
    if rc:
        raise ValueError("oracle matmul_integer: unsupported zero points or batch")
    return out.reshape(bs + [m, n])


def qlinear_multiplier(a_scale, b_scale, y_scale):
    return np.float32(_load().orc_qlinear_multiplier(float(a_scale), float(b_scale), float(y_scale)))


def round_even(v):
    return int(_load().orc_round_even(float(v)))


def dynamic_quantize_linear(x):
    """``opDynamicQuantizeLinear`` (onnx_ops.dart:3556-3583): returns
    (y uint8 of x's shape, scale float32, zero point int)."""
    x = _c(x, np.float32)
    y = np.zeros(x.size, np.uint8)
    sc = ctypes.c_float()
    zp = _load().orc_dynamic_quantize_linear(_p(x.reshape(-1), _f32p), x.size, _p(y, _u8p), ctypes.byref(sc))
    return y.reshape(x.shape), np.float32(sc.value), int(zp)


def qlinear_matmul(a, a_scale, a_zp, b, b_scale, b_zp, y_scale, y_zp, lo, hi, nthreads=1):
    """``opQLinearMatMul`` (onnx_qlinear_ops.dart:85-108); int64 result."""
    a32, b32, az, bz, m, k, n, ab, bb, bs = _int_operands(a, b, a_zp, b_zp)
    out = np.zeros(max(ab, bb) * m * n, np.int64)
    yz = 0 if y_zp is None else int(np.asarray(y_zp).reshape(-1)[0])
    rc = _load().orc_qlinear_matmul(_p(a32, _i32p), ab, m, k, _p(b32, _i32p), bb, n, _p(az, _i32p),
                                    0 if az is None else az.size, _p(bz, _i32p), 0 if bz is None else bz.size,
                                    float(np.float32(a_scale)), float(np.float32(b_scale)),
                                    float(np.float32(y_scale)), yz, lo, hi, _p(out, _i64p), nthreads)
    if rc:
        raise ValueError("oracle qlinear_matmul: unsupported zero points or batch")
    return out.reshape(bs + [m, n])


def matmul_nbits(a, b_q, scales, zero_points, k, n, block_size, bias=None, nthreads=1):
    """``opMatMulNBits`` (onnx_qlinear_ops.dart:115-228), bits=4.

    ``zero_points`` may be packed uint8 (uint4 pairs), float32, or None."""
    a = _c(a, np.float32)
    m = a.size // k
    bq = _c(np.asarray(b_q).reshape(-1), np.uint8)
    sc = _c(np.asarray(scales).reshape(-1), np.float32)
    zu = zf = None
    if zero_points is not None:
        zp = np.asarray(zero_points)
        if zp.dtype == np.uint8:
            zu = _c(zp.reshape(-1), np.uint8)
        else:
            zf = _c(zp.reshape(-1), np.float32)
    bi = None if bias is None else _c(np.asarray(bias).reshape(-1), np.float32)
    out = np.zeros(m * n, np.float32)
    rc = _load().orc_matmul_nbits(_p(a, _f32p), m, k, _p(bq, _u8p), _p(sc, _f32p), _p(zu, _u8p), _p(zf, _f32p),
                                  _p(bi, _f32p), n, block_size, _p(out, _f32p), nthreads)
    if rc:
        raise ValueError("oracle matmul_nbits: invalid K, N or block_size")
    return out.reshape(list(a.shape[:-1]) + [n])


def nbits_dequant(b_q, scales, zero_points, k, n, block_size):
    """Float32 weights W[n, k] exactly as the reference's ``weight()`` makes them."""
    bq = _c(np.asarray(b_q).reshape(-1), np.uint8)
    sc = _c(np.asarray(scales).reshape(-1), np.float32)
    zu = zf = None
    if zero_points is not None:
        zp = np.asarray(zero_points)
        if zp.dtype == np.uint8:
            zu = _c(zp.reshape(-1), np.uint8)
        else:
            zf = _c(zp.reshape(-1), np.float32)
    w = np.zeros(n * k, np.float32)
    _load().orc_nbits_dequant(_p(bq, _u8p), _p(sc, _f32p), _p(zu, _u8p), _p(zf, _f32p), k, n, block_size,
                              _p(w, _f32p))
    return w.reshape(n, k)


# ---------------------------------------------------------------------------
# Conv / ConvInteger / QLinearConv
# ---------------------------------------------------------------------------

def resolve_pads(in_sp, kernel, strides, dilations, auto_pad="NOTSET", pads=None):
    """``_resolvePads`` (lib/src/onnx_nn_ops.dart:38-88) without ceil mode:
    (pads [begin..., end...], output spatial dims)."""
    nd = len(in_sp)
    p, out = [0] * (2 * nd), [0] * nd
    for k in range(nd):
        window = dilations[k] * (kernel[k] - 1) + 1
        if auto_pad in ("SAME_UPPER", "SAME_LOWER"):
            out[k] = (in_sp[k] + strides[k] - 1) // strides[k]
            total = max(0, (out[k] - 1) * strides[k] + window - in_sp[k])
            small = total // 2
            p[k] = small if auto_pad == "SAME_UPPER" else total - small
            p[nd + k] = total - p[k]
        elif auto_pad == "VALID":
            out[k] = (in_sp[k] - window) // strides[k] + 1
        else:
            p[k] = 0 if pads is None else int(pads[k])
            p[nd + k] = 0 if pads is None else int(pads[nd + k])
            out[k] = (in_sp[k] + p[k] + p[nd + k] - window) // strides[k] + 1
    return p, out


def conv_winograd_eligible(w_shape, in_shape, strides=None, pads=None, dilations=None, group=1,
                           auto_pad="NOTSET", min_out_pixels=1024):
    """``convWinogradEligible`` (lib/src/onnx_nn_ops.dart:779-812): whether the
    executor takes opConv's Winograd F(2x2, 3x3) branch for an initializer
    weight of this shape (the executor also requires the weight to be an
    initializer, onnx_graph.dart:2450-2454)."""
    if group != 1 or len(w_shape) != 4 or len(in_shape) != 4:
        return False
    if w_shape[2] != 3 or w_shape[3] != 3:
        return False
    if auto_pad != "NOTSET" or pads is None or len(pads) != 4:
        return False
    if not (all(v == 0 for v in pads) or all(v == 1 for v in pads)):
        return False
    s = list(strides) if strides is not None else [1, 1]
    d = list(dilations) if dilations is not None else [1, 1]
    if len(s) != 2 or len(d) != 2 or s != [1, 1] or d != [1, 1]:
        return False
    _, osp = resolve_pads(list(in_shape[2:]), [3, 3], s, d, auto_pad, list(pads))
    return osp[0] * osp[1] >= min_out_pixels


def conv_winograd_f32(x, w, bias=None, pad=1):
    """opConv's Winograd F(2x2, 3x3) branch (lib/src/onnx_nn_ops.dart:271-293
    with pretransformWinogradF2x2 :584-628 and _convWinogradF2x2 :630-748), a
    standalone call: x [N, C, H, W], w [M, C, 3, 3], pads all `pad` (0 or 1),
    stride and dilation 1."""
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    bias = _c(bias, np.float32)
    n, c, h, wd = x.shape
    m = w.shape[0]
    if w.shape != (m, c, 3, 3):
        raise ValueError("oracle winograd conv: weight must be [M, C, 3, 3]")
    out = np.zeros((n, m, h + 2 * pad - 2, wd + 2 * pad - 2), np.float32)
    rc = _load().orc_conv_winograd_f2x2(_p(x, _f32p), n, c, h, wd, _p(w, _f32p), m, _p(bias, _f32p), int(pad),
                                        _p(out, _f32p))
    if rc:
        raise ValueError(f"oracle winograd conv: bad arguments ({rc})")
    return out


def conv_f32(x, w, bias=None, strides=None, pads=None, dilations=None, group=1, auto_pad="NOTSET"):
    """``opConv`` (lib/src/onnx_nn_ops.dart:179-545) outside its Winograd
    branch: im2col + matmulKernel for 1-D / 2-D, double accumulation for
    depthwise 2-D and for 3-D."""
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    bias = _c(bias, np.float32)
    nd = x.ndim - 2
    kernel = list(w.shape[2:])
    s = list(strides) if strides is not None else [1] * nd
    d = list(dilations) if dilations is not None else [1] * nd
    p, osp = resolve_pads(list(x.shape[2:]), kernel, s, d, auto_pad, pads)
    out = np.zeros([x.shape[0], w.shape[0]] + osp, np.float32)
    arr = lambda v: np.array(v, np.int64)
    xs, ks, ss, ps, ds = arr(x.shape), arr(kernel), arr(s), arr(p), arr(d)
    rc = _load().orc_conv_f32(_p(x, _f32p), _p(xs, _i64p), nd, _p(w, _f32p), _p(ks, _i64p), w.shape[0],
                              _p(bias, _f32p), _p(ss, _i64p), _p(ps, _i64p), _p(ds, _i64p), int(group),
                              _p(out, _f32p))
    if rc:
        raise ValueError(f"oracle conv: bad arguments ({rc})")
    return out


def _conv_int(x, w, x_zp, w_zp, strides, pads, dilations, group):
    """``_convIntAcc`` with opConvInteger's 1-D reshape (:305-320)."""
    x = np.asarray(x)
    w = np.asarray(w)
    if x.ndim == 3:
        x = x.reshape(x.shape[0], x.shape[1], 1, x.shape[2])
        w = w.reshape(w.shape[0], w.shape[1], 1, w.shape[2])
        strides = [1, 1 if strides is None else strides[0]]
        pads = None if pads is None else [0, pads[0], 0, pads[1]]
        dilations = [1, 1 if dilations is None else dilations[0]]
        one_d = True
    else:
        one_d = False
    s = strides or [1, 1]
    p = pads or [0, 0, 0, 0]
    d = dilations or [1, 1]
    m = w.shape[0]
    osp = [(x.shape[2 + a] + p[a] + p[2 + a] - (d[a] * (w.shape[2 + a] - 1) + 1)) // s[a] + 1 for a in range(2)]
    wz = np.zeros(m, np.int32) if w_zp is None else np.broadcast_to(
        np.asarray(w_zp).astype(np.int32).ravel()[:1] if np.asarray(w_zp).size == 1 else
        np.asarray(w_zp).astype(np.int32).ravel(), (m,)).copy()
    xz = 0 if x_zp is None else int(np.asarray(x_zp).ravel()[0])
    xi = np.ascontiguousarray(x, dtype=np.int32)
    wi = np.ascontiguousarray(w, dtype=np.int32)
    acc = np.zeros([x.shape[0], m] + osp, np.int64)
    _load().orc_conv_int_acc(_p(xi, _i32p), x.shape[0], x.shape[1], x.shape[2], x.shape[3], _p(wi, _i32p), m,
                             w.shape[1], w.shape[2], w.shape[3], xz, _p(wz, _i32p), s[0], s[1], d[0], d[1], p[0],
                             p[1], int(group), osp[0], osp[1], _p(acc, _i64p))
    return acc, one_d


def conv_integer(x, w, x_zp=None, w_zp=None, strides=None, pads=None, dilations=None, group=1):
    """``opConvInteger`` (lib/src/onnx_qlinear_ops.dart:305-338): int32-exact
    accumulators (int64 here, as in the reference)."""
    if w_zp is not None and np.asarray(w_zp).size not in (1, np.asarray(w).shape[0]):
        raise NotImplementedError("ConvInteger: weight zero point must be scalar or per-output-channel")
    acc, one_d = _conv_int(x, w, x_zp, w_zp, strides, pads, dilations, group)
    return acc.reshape(acc.shape[0], acc.shape[1], acc.shape[3]) if one_d else acc


def qlinear_conv(x, x_scale, x_zp, w, w_scale, w_zp, y_scale, y_zp, bias=None, strides=None, pads=None,
                 dilations=None, group=1, lo=0, hi=255):
    """``opQLinearConv`` (lib/src/onnx_qlinear_ops.dart:341-382), 2-D."""
    acc, _ = _conv_int(x, w, x_zp, w_zp, strides, pads, dilations, group)
    n, m = acc.shape[0], acc.shape[1]
    spn = int(np.prod(acc.shape[2:]))
    ws = np.ascontiguousarray(np.asarray(w_scale, np.float32).astype(np.float64).ravel())
    b = None if bias is None else np.ascontiguousarray(np.asarray(bias).astype(np.int64).ravel())
    yz = 0 if y_zp is None else int(np.asarray(y_zp).ravel()[0])
    out = np.zeros(acc.shape, np.int64)
    acc = np.ascontiguousarray(acc)
    _load().orc_qlinear_conv_requant(_p(acc, _i64p), n, m, spn, float(np.float32(np.asarray(x_scale).ravel()[0])),
                                     ws.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), ws.size,
                                     float(np.float32(np.asarray(y_scale).ravel()[0])), yz, _p(b, _i64p), lo, hi,
                                     _p(out, _i64p))
    return out


def conv_transpose_f32(x, w, bias=None, strides=None, pads=None, dilations=None, output_padding=None,
                       output_shape=None, group=1):
    """``opConvTranspose`` (lib/src/onnx_nn_ops.dart:815-1060): the GEMM +
    overlap-add path for one image of 1-D / 2-D without output_shape, the
    generic double-product scatter otherwise."""
    x = _c(x, np.float32)
    w = _c(w, np.float32)
    bias = _c(bias, np.float32)
    nd = x.ndim - 2
    arr = lambda v: np.array(v, np.int64)
    ks = arr(w.shape[2:])
    st = arr(strides if strides is not None else [1] * nd)
    dl = arr(dilations if dilations is not None else [1] * nd)
    op = arr(output_padding if output_padding is not None else [0] * nd)
    pd = None if pads is None else arr(pads)
    osh = None if output_shape is None else arr(list(output_shape)[-nd:])
    mpg = w.shape[1]
    out = np.zeros(x.shape[0] * mpg * group * 4 * int(np.prod([
        (x.shape[2 + a] - 1) * st[a] + dl[a] * (ks[a] - 1) + 1 + op[a] for a in range(nd)])) + 16, np.float32)
    osp = np.zeros(3, np.int64)
    xs = arr(x.shape)
    rc = _load().orc_conv_transpose_f32(_p(x, _f32p), _p(xs, _i64p), nd, _p(w, _f32p), _p(ks, _i64p), mpg,
                                        int(group), _p(bias, _f32p), _p(st, _i64p), _p(pd, _i64p), _p(dl, _i64p),
                                        _p(op, _i64p), _p(osh, _i64p), _p(out, _f32p), _p(osp, _i64p))
    if rc:
        raise ValueError(f"oracle conv_transpose: bad arguments ({rc})")
    shape = [x.shape[0], mpg * group] + [int(v) for v in osp[:nd]]
    return out[:int(np.prod(shape))].reshape(shape).copy()
