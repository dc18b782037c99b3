"""The MatMul-family operators, mirroring the reference's op functions.

Same names, argument meaning and error behaviour as
  opMatMul         lib/src/onnx_ops.dart:1710-1766
  opGemm           lib/src/onnx_ops.dart:2152-2173
  opMatMulInteger  lib/src/onnx_qlinear_ops.dart:32-81
  opQLinearMatMul  lib/src/onnx_qlinear_ops.dart:85-108
  opMatMulNBits    lib/src/onnx_qlinear_ops.dart:115-228
  opConv           lib/src/onnx_nn_ops.dart:179-545
  opConvInteger    lib/src/onnx_qlinear_ops.dart:305-338
  opQLinearConv    lib/src/onnx_qlinear_ops.dart:341-382
  opConvTranspose  lib/src/onnx_nn_ops.dart:815-1060
but executed by libb200mm.so on the GPU. Operands may be numpy arrays (host
values, uploaded for the call), DeviceTensor (device-resident, e.g. the output
of a previous op), or — for the weight operand — a PackedWeight prepared once
at session load. Results are DeviceTensor; `.numpy()` downloads them.

There is no CPU fallback: without the CUDA library or a B200 the calls raise.
MatMulInteger / QLinearMatMul results come back as int32 / uint8 / int8 device
tensors (ONNX types); `as_reference_int64` converts a downloaded result to
the int64 storage the reference's Tensor.int64 uses.
"""
from __future__ import annotations

import ctypes
import threading

import numpy as np

from . import _native as N
from .runtime import Context, DeviceTensor, PackedWeight

MODE_EXACT = N.MODE_EXACT
MODE_FAST = N.MODE_FAST
MODE_PRECISE = N.MODE_PRECISE

_default = {}
_lock = threading.Lock()


def default_context(device: int = 0) -> Context:
    with _lock:
        ctx = _default.get(device)
        if ctx is None or ctx.handle is None:
            ctx = Context(device)
            _default[device] = ctx
        return ctx


def _ctx(ctx):
    return ctx if ctx is not None else default_context()


def _dev(ctx: Context, x, dtype=None):
    """Device handle for an operand (None stays None)."""
    if x is None:
        return None, None
    if isinstance(x, DeviceTensor):
        return x.handle, x
    arr = np.asarray(x) if dtype is None else np.asarray(x, dtype)
    t = ctx.upload(arr)
    return t.handle, t


def _out(out):
    h = ctypes.c_void_p(out.handle.value if out is not None else None)
    return h


def _wrap_out(ctx, h, out):
    return out if out is not None else DeviceTensor(ctx, h)


def _shape(x):
    return list(x.shape)


def as_reference_int64(y) -> np.ndarray:
    """Host int64 copy, the storage the reference's Tensor.int64 uses."""
    arr = y.numpy() if isinstance(y, DeviceTensor) else np.asarray(y)
    return arr.astype(np.int64)


# ---------------------------------------------------------------------------
# fp32
# ---------------------------------------------------------------------------

def opMatMul(a, b, *, mode: int = MODE_EXACT, ctx: Context | None = None, out: DeviceTensor | None = None):
    """numpy-style matmul: last two dims are the matrix dims, leading dims
    batch (broadcastable). `b` may be a PackedWeight (2-D initializer)."""
    ctx = _ctx(ctx)
    ah, _a = _dev(ctx, a, np.float32)
    if isinstance(b, PackedWeight):
        bh, bw, _b = None, b.handle, None
    else:
        bh, _b = _dev(ctx, b, np.float32)
        bw = None
    y = _out(out)
    N.check(ctx.lib.b2m_matmul_f32(ctx.handle, ah, bh, bw, int(mode), ctypes.byref(y)))
    return _wrap_out(ctx, y, out)


def opGemm(a, b, c=None, *, alpha: float = 1.0, beta: float = 1.0, transA: bool = False, transB: bool = False,
           mode: int = MODE_EXACT, ctx: Context | None = None, out: DeviceTensor | None = None):
    """Gemm: Y = alpha * A' * B' + beta * C (A'/B' optionally transposed)."""
    ctx = _ctx(ctx)
    ah, _a = _dev(ctx, a, np.float32)
    if isinstance(b, PackedWeight):
        bh, bw, _b = None, b.handle, None
    else:
        bh, _b = _dev(ctx, b, np.float32)
        bw = None
    ch, _c = _dev(ctx, c, np.float32)
    y = _out(out)
    N.check(ctx.lib.b2m_gemm_f32(ctx.handle, ah, bh, bw, ch, float(np.float32(alpha)), float(np.float32(beta)),
                                 1 if transA else 0, 1 if transB else 0, int(mode), ctypes.byref(y)))
    return _wrap_out(ctx, y, out)


# ---------------------------------------------------------------------------
# int8
# ---------------------------------------------------------------------------

def _int_operand(ctx, x):
    if x is None:
        return None, None
    if isinstance(x, DeviceTensor):
        return x.handle, x
    arr = np.asarray(x)
    if arr.dtype not in (np.uint8, np.int8):
        raise N.ArgumentError(f"integer operand must be uint8 or int8, got {arr.dtype}")
    return _dev(ctx, arr)


def opMatMulInteger(a, b, aZp=None, bZp=None, *, ctx: Context | None = None, out: DeviceTensor | None = None):
    """`y_int32 = (A - aZp) . (B - bZp)`; zero points scalar, per-row [M] for
    A or per-column [N] for B. `b` may be a PackedWeight."""
    ctx = _ctx(ctx)
    ah, _a = _int_operand(ctx, a)
    if isinstance(b, PackedWeight):
        bh, bw, _b = None, b.handle, None
    else:
        (bh, _b), bw = _int_operand(ctx, b), None
    azh, _az = _int_operand(ctx, aZp)
    bzh, _bz = _int_operand(ctx, bZp)
    y = _out(out)
    N.check(ctx.lib.b2m_matmul_integer(ctx.handle, ah, bh, bw, azh, bzh, ctypes.byref(y)))
    return _wrap_out(ctx, y, out)


def _scalar(x, what):
    arr = np.asarray(x.numpy() if isinstance(x, DeviceTensor) else x)
    if arr.size != 1:
        raise N.UnsupportedError("QLinearMatMul: only per-tensor scales supported")
    return arr.reshape(-1)[0]


def opQLinearMatMul(a, aS, aZp, b, bS, bZp, yS, yZp, *, lo: int, hi: int, ctx: Context | None = None,
                    out: DeviceTensor | None = None):
    """MatMulInteger + requantize with aS*bS/yS, saturating to [lo, hi]
    (lo/hi come from the output zero point's dtype)."""
    ctx = _ctx(ctx)
    a_s, b_s, y_s = (float(np.float32(_scalar(v, n))) for v, n in ((aS, "aS"), (bS, "bS"), (yS, "yS")))
    yz = 0 if yZp is None else int(_scalar(yZp, "yZp"))
    ah, _a = _int_operand(ctx, a)
    if isinstance(b, PackedWeight):
        bh, bw, _b = None, b.handle, None
    else:
        (bh, _b), bw = _int_operand(ctx, b), None
    azh, _az = _int_operand(ctx, aZp)
    bzh, _bz = _int_operand(ctx, bZp)
    y = _out(out)
    N.check(ctx.lib.b2m_qlinear_matmul(ctx.handle, ah, a_s, azh, bh, bw, b_s, bzh, y_s, yz, int(lo), int(hi),
                                       ctypes.byref(y)))
    return _wrap_out(ctx, y, out)


def opDynamicQuantizeLinear(x, *, ctx: Context | None = None):
    """opDynamicQuantizeLinear (lib/src/onnx_ops.dart:3556): returns
    [y uint8 (x's shape), scale float32 scalar, zero point uint8 scalar], all
    device tensors, bit-exact with the reference. y and the zero point feed
    opMatMulInteger as A and aZp without leaving the device."""
    ctx = _ctx(ctx)
    if isinstance(x, DeviceTensor):
        xt = x
    else:
        xt = ctx.upload(np.asarray(x, np.float32))
    if xt.dtype != np.float32:
        raise N.ArgumentError("DynamicQuantizeLinear: x must be float32")
    shape = xt.shape
    n = int(np.prod(shape)) if shape else 1
    y = ctx.empty(shape, np.uint8)
    scale = ctx.empty([], np.float32)
    zp = ctx.empty([], np.uint8)
    N.check(ctx.lib.b2m_dynamic_quantize_linear_dev(ctx.handle, ctypes.c_void_p(xt.data_ptr), n,
                                                    ctypes.c_void_p(y.data_ptr), ctypes.c_void_p(scale.data_ptr),
                                                    ctypes.c_void_p(zp.data_ptr)))
    return [y, scale, zp]


# ---------------------------------------------------------------------------
# int4 MatMulNBits
# ---------------------------------------------------------------------------

def _is_float(x):
    return np.dtype(x.dtype).kind == "f"


def validate_nbits(a_shape, a_dtype, bQ, scales, zeroPoints, bias, k, n, bits, blockSize):
    """The reference's checks, in its order and with its messages
    (onnx_qlinear_ops.dart:126-166)."""
    if bits != 4:
        raise N.UnsupportedError(f"MatMulNBits: only bits=4 supported, got {bits}")
    if (k <= 0 or n <= 0 or blockSize < 16 or (blockSize & (blockSize - 1)) != 0 or len(a_shape) < 1
            or a_shape[-1] != k):
        raise N.ArgumentError("MatMulNBits: invalid K, N, block_size or input shape")
    n_blocks = (k + blockSize - 1) // blockSize
    blob = blockSize // 2
    zp_stride = (n_blocks + 1) // 2
    if isinstance(bQ, PackedWeight):
        raise N.ArgumentError("MatMulNBits: pass raw initializers to validate_nbits")
    bq_shape = _shape(bQ)
    sc_shape = _shape(scales)
    if (len(bq_shape) != 3 or bq_shape[0] != n or bq_shape[1] != n_blocks or bq_shape[2] != blob
            or np.dtype(bQ.dtype) != np.uint8 or np.dtype(a_dtype).kind != "f" or not _is_float(scales)
            or int(np.prod(sc_shape)) != n * n_blocks or len(sc_shape) not in (1, 2)
            or (len(sc_shape) == 2 and (sc_shape[0] != n or sc_shape[1] != n_blocks))):
        raise N.ArgumentError("MatMulNBits: invalid packed weights or scales")
    if zeroPoints is not None:
        zs = _shape(zeroPoints)
        packed = np.dtype(zeroPoints.dtype) == np.uint8
        if (len(zs) not in (1, 2) or (len(zs) == 2 and zs[0] != n)
                or (int(np.prod(zs)) != n * zp_stride if packed
                    else (not _is_float(zeroPoints) or int(np.prod(zs)) != n * n_blocks))):
            raise N.ArgumentError("MatMulNBits: invalid zero_points")
    if bias is not None:
        bs = _shape(bias)
        if not _is_float(bias) or len(bs) != 1 or bs[0] != n:
            raise N.ArgumentError("MatMulNBits: bias must be floating point [N]")


def prepack_nbits(ctx: Context, bQ, scales, zeroPoints, *, k, n, bits, blockSize) -> PackedWeight:
    return ctx.prepack_nbits(np.asarray(bQ), np.asarray(scales),
                             None if zeroPoints is None else np.asarray(zeroPoints), k, n, bits, blockSize)


def opMatMulNBits(a, bQ, scales=None, zeroPoints=None, *, k: int, n: int, bits: int = 4, blockSize: int,
                  bias=None, mode: int = MODE_FAST, ctx: Context | None = None, out: DeviceTensor | None = None):
    """`y = A . dequant(B)^T (+ bias)`, B block-quantized to 4 bits.

    `bQ` is the packed uint8 [N, ceil(K/block), block/2] initializer (with
    `scales` and optional `zeroPoints`), or a PackedWeight from
    `prepack_nbits`. mode FAST (default) runs the tensor-core kernels on f16
    weights and activations; mode PRECISE splits both into two bf16 terms
    (three tensor-core products, ~1e-5 relative) for long chains; mode EXACT
    reproduces the reference bit for bit."""
    ctx = _ctx(ctx)
    a_shape = _shape(a)
    a_dtype = a.dtype
    if isinstance(bQ, PackedWeight):
        if bits != 4:
            raise N.UnsupportedError(f"MatMulNBits: only bits=4 supported, got {bits}")
        kk, nn = bQ.kn
        if kk != k or nn != n or len(a_shape) < 1 or a_shape[-1] != k:
            raise N.ArgumentError("MatMulNBits: invalid K, N, block_size or input shape")
        if bias is not None and (not _is_float(bias) or len(_shape(bias)) != 1 or _shape(bias)[0] != n):
            raise N.ArgumentError("MatMulNBits: bias must be floating point [N]")
        w = bQ
    else:
        validate_nbits(a_shape, a_dtype, np.asarray(bQ), np.asarray(scales),
                       None if zeroPoints is None else np.asarray(zeroPoints),
                       None if bias is None or isinstance(bias, DeviceTensor) else np.asarray(bias),
                       k, n, bits, blockSize)
        w = prepack_nbits(ctx, bQ, scales, zeroPoints, k=k, n=n, bits=bits, blockSize=blockSize)
    ah, _a = _dev(ctx, a, np.float32)
    bh, _b = _dev(ctx, bias, np.float32)
    y = _out(out)
    N.check(ctx.lib.b2m_matmul_nbits(ctx.handle, ah, w.handle, bh, int(mode), ctypes.byref(y)))
    return _wrap_out(ctx, y, out)


# ---------------------------------------------------------------------------
# Convolutions through the GEMM cores
# ---------------------------------------------------------------------------

AUTO_PAD = {"NOTSET": 0, "SAME_UPPER": 1, "SAME_LOWER": 2, "VALID": 3}


def _i64_array(v, count=None, what=""):
    if v is None:
        return None, None
    arr = np.ascontiguousarray(np.asarray(v, np.int64).ravel())
    if count is not None and arr.size != count:
        raise N.ArgumentError(f"Conv: {what} must have {count} values, got {arr.size}")
    return arr, arr.ctypes.data_as(ctypes.c_void_p)


def _spatial_attrs(pw, strides, pads, dilations):
    """kernel_shape / strides / pads / dilations arrays of the lengths the
    C ABI reads (nd, nd, 2 nd, nd)."""
    nd = len(pw.shape) - 2
    return (_i64_array(pw.shape[2:]), _i64_array(strides, nd, "strides"), _i64_array(pads, 2 * nd, "pads"),
            _i64_array(dilations, nd, "dilations"))


def _conv_weight(ctx, w):
    if isinstance(w, PackedWeight):
        if w.shape is None:
            raise N.ArgumentError("Conv: the packed weight was not made by prepack_conv")
        return w, None
    pw = ctx.prepack_conv(np.asarray(w.numpy() if isinstance(w, DeviceTensor) else w))
    return pw, pw


def _check_conv_rank(x, pw, lo, hi):
    """The weight's spatial rank must match the input's (opConv asserts
    w.rank == x.rank, onnx_nn_ops.dart:197); ranks outside [lo, hi] are left
    to the library, which rejects them as unsupported."""
    xr = len(x.shape) if hasattr(x, "shape") else np.ndim(x)
    if lo <= xr <= hi and len(pw.shape) != xr:
        raise N.ArgumentError("Conv weight rank must match input rank")


def opConv(x, w, bias=None, *, strides=None, pads=None, dilations=None, group: int = 1, autoPad: str = "NOTSET",
           mode: int = MODE_EXACT, ctx: Context | None = None, out: DeviceTensor | None = None):
    """Conv over 1-3 spatial dims: x [N][C][spatial...], w [M][C/group][kernel...]
    (a PackedWeight from Context.prepack_conv, or a host array packed for the
    call), bias [M]. Pads are [begin..., end...] as the ONNX attribute."""
    ctx = _ctx(ctx)
    if autoPad not in AUTO_PAD:
        raise N.ArgumentError(f"Conv: unknown auto_pad {autoPad!r}")
    pw, tmp = _conv_weight(ctx, w)
    _check_conv_rank(x, pw, 3, 5)
    xh, _x = _dev(ctx, x, np.float32)
    bh, _b = _dev(ctx, bias, np.float32)
    (ks, ksp), (st, stp), (pd, pdp), (dl, dlp) = _spatial_attrs(pw, strides, pads, dilations)
    y = _out(out)
    try:
        N.check(ctx.lib.b2m_conv_f32(ctx.handle, xh, pw.handle, bh, ksp, stp, pdp, dlp, int(group), AUTO_PAD[autoPad],
                                     int(mode), ctypes.byref(y)))
    finally:
        if tmp is not None:
            ctx.synchronize()
            tmp.free()
    return _wrap_out(ctx, y, out)


def opConvInteger(x, w, xZp=None, wZp=None, *, strides=None, pads=None, dilations=None, group: int = 1,
                  ctx: Context | None = None, out: DeviceTensor | None = None):
    """ConvInteger (1-D / 2-D): int32 y = sum over taps of (x - xZp)(w - wZp[m])."""
    ctx = _ctx(ctx)
    pw, tmp = _conv_weight(ctx, w)
    _check_conv_rank(x, pw, 3, 4)
    xh, _x = _int_operand(ctx, x)
    xzh, _xz = _int_operand(ctx, xZp)
    wzh, _wz = _int_operand(ctx, wZp)
    (ks, ksp), (st, stp), (pd, pdp), (dl, dlp) = _spatial_attrs(pw, strides, pads, dilations)
    y = _out(out)
    try:
        N.check(ctx.lib.b2m_conv_integer(ctx.handle, xh, xzh, pw.handle, wzh, ksp, stp, pdp, dlp, int(group),
                                         ctypes.byref(y)))
    finally:
        if tmp is not None:
            ctx.synchronize()
            tmp.free()
    return _wrap_out(ctx, y, out)


def opQLinearConv(x, xS, xZp, w, wS, wZp, yS, yZp, bias=None, *, strides=None, pads=None, dilations=None,
                  group: int = 1, lo: int, hi: int, ctx: Context | None = None, out: DeviceTensor | None = None):
    """QLinearConv (2-D): ConvInteger's accumulator plus the int32 bias,
    requantized per output channel with xS * wS[c] / yS in double, rounded half
    to even, shifted by yZp and clamped to [lo, hi] (from yZp's dtype)."""
    ctx = _ctx(ctx)
    pw, tmp = _conv_weight(ctx, w)
    _check_conv_rank(x, pw, 4, 4)
    host = lambda v: np.asarray(v.numpy() if isinstance(v, DeviceTensor) else v)
    xs = float(np.float32(host(xS).reshape(-1)[0]))
    ys = float(np.float32(host(yS).reshape(-1)[0]))
    yz = 0 if yZp is None else int(host(yZp).reshape(-1)[0])
    wsh, _ws = _dev(ctx, wS, np.float32)
    xh, _x = _int_operand(ctx, x)
    xzh, _xz = _int_operand(ctx, xZp)
    wzh, _wz = _int_operand(ctx, wZp)
    bh, _b = _dev(ctx, bias, np.int32)
    (ks, ksp), (st, stp), (pd, pdp), (dl, dlp) = _spatial_attrs(pw, strides, pads, dilations)
    y = _out(out)
    try:
        N.check(ctx.lib.b2m_qlinear_conv(ctx.handle, xh, xs, xzh, pw.handle, wsh, wzh, ys, yz, bh, ksp, stp, pdp, dlp, int(group), int(lo), int(hi),
                                         ctypes.byref(y)))
    finally:
        if tmp is not None:
            ctx.synchronize()
            tmp.free()
    return _wrap_out(ctx, y, out)


def opConvTranspose(x, w, bias=None, *, strides=None, pads=None, dilations=None, outputPadding=None,
                    outputShape=None, group: int = 1, ctx: Context | None = None, out: DeviceTensor | None = None):
    """ConvTranspose over 1-3 spatial dims: x [N][C][spatial...], w
    [C][M/group][kernel...] (host array or DeviceTensor), bias [M]. Pads are
    [begin..., end...]; output_shape lists the spatial dims (or the full
    N, C, spatial shape, of which the last nd entries are used)."""
    ctx = _ctx(ctx)
    xh, _x = _dev(ctx, x, np.float32)
    wh, _w = _dev(ctx, w, np.float32)
    bh, _b = _dev(ctx, bias, np.float32)
    xr = len(x.shape) if hasattr(x, "shape") else np.ndim(x)
    nd = xr - 2
    if 1 <= nd <= 3:
        st, stp = _i64_array(strides, nd, "strides")
        pd, pdp = _i64_array(pads, 2 * nd, "pads")
        dl, dlp = _i64_array(dilations, nd, "dilations")
        op, opp = _i64_array(outputPadding, nd, "output_padding")
        osh, oshp = _i64_array(None if outputShape is None else list(outputShape)[-nd:], nd, "output_shape")
    else:
        stp = pdp = dlp = opp = oshp = None
    y = _out(out)
    N.check(ctx.lib.b2m_conv_transpose_f32(ctx.handle, xh, wh, bh, stp, pdp, dlp, opp, oshp, int(group),
                                           ctypes.byref(y)))
    return _wrap_out(ctx, y, out)
