"""Host-side objects over the C ABI: Context, DeviceTensor, PackedWeight.

DeviceTensor is the device-resident counterpart of the reference's Tensor
(lib/src/tensor.dart:16-223): a dtype, a row-major shape and a buffer — here
a device buffer owned by the library (or borrowed from the caller, e.g. a
torch tensor, via `wrap`). PackedWeight holds an initializer prepacked once
at session load (the reference's `_prepackedGemmB` cache,
lib/src/onnx_graph.dart:102-105).
"""
from __future__ import annotations

import contextlib
import ctypes

import numpy as np

from . import _native as N

_NP_TO_B2M = {
    np.dtype(np.float32): N.B2M_FLOAT,
    np.dtype(np.uint8): N.B2M_UINT8,
    np.dtype(np.int8): N.B2M_INT8,
    np.dtype(np.int32): N.B2M_INT32,
    np.dtype(np.int64): N.B2M_INT64,
    np.dtype(np.float16): N.B2M_FLOAT16,
}
_B2M_TO_NP = {v: k for k, v in _NP_TO_B2M.items()}


def b2m_dtype(dt) -> int:
    try:
        return _NP_TO_B2M[np.dtype(dt)]
    except KeyError:
        raise N.ArgumentError(f"unsupported dtype {dt}") from None


def np_dtype(code: int):
    return _B2M_TO_NP[code]


def _shape_arr(shape):
    arr = (ctypes.c_int64 * max(1, len(shape)))(*[int(s) for s in shape])
    return arr


class Context:
    """One device, one stream, one memory pool (b2m_init / b2m_shutdown)."""

    def __init__(self, device: int = 0, library: str | None = None):
        self.lib = N.load(library)
        h = ctypes.c_void_p()
        N.check(self.lib.b2m_init(int(device), ctypes.byref(h)))
        self.handle = h
        self.device = int(device)
        self._cancel = ctypes.c_int32(0)

    # -- lifecycle ---------------------------------------------------------
    def close(self):
        if getattr(self, "handle", None):
            N.check(self.lib.b2m_shutdown(self.handle))
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # -- control -----------------------------------------------------------
    def set_stream(self, stream_ptr: int | None):
        N.check(self.lib.b2m_set_stream(self.handle, ctypes.c_void_p(stream_ptr or 0)))

    def synchronize(self):
        N.check(self.lib.b2m_synchronize(self.handle))

    def enable_cancel_flag(self):
        """Routes the context's cancel flag to `self.cancel()` (checkpoint-style)."""
        N.check(self.lib.b2m_set_cancel_flag(self.handle, ctypes.byref(self._cancel)))

    def cancel(self, on: bool = True):
        self._cancel.value = 1 if on else 0

    def set_byte_budget(self, nbytes: int):
        N.check(self.lib.b2m_set_byte_budget(self.handle, int(nbytes)))

    def set_attention_mode(self, mode: int):
        """N.MODE_EXACT: fp32 CUDA-core attention with no key splits (each
        sequence's result independent of the batch); N.MODE_FAST (default):
        the tensor-core kernels."""
        N.check(self.lib.b2m_set_attention_mode(self.handle, int(mode)))

    def enable_timing(self, on: bool = True):
        N.check(self.lib.b2m_enable_timing(self.handle, 1 if on else 0))

    def last_kernel_ms(self) -> float:
        ms = ctypes.c_float()
        N.check(self.lib.b2m_last_kernel_ms(self.handle, ctypes.byref(ms)))
        return float(ms.value)

    # -- tensors -----------------------------------------------------------
    def empty(self, shape, dtype=np.float32) -> "DeviceTensor":
        h = ctypes.c_void_p()
        N.check(self.lib.b2m_tensor_alloc(self.handle, b2m_dtype(dtype), _shape_arr(shape), len(shape),
                                          ctypes.byref(h)))
        return DeviceTensor(self, h)

    def upload(self, arr) -> "DeviceTensor":
        arr = np.ascontiguousarray(arr)
        t = self.empty(arr.shape, arr.dtype)
        N.check(self.lib.b2m_tensor_upload(self.handle, t.handle, arr.ctypes.data_as(ctypes.c_void_p), arr.nbytes))
        return t

    def wrap(self, device_ptr: int, shape, dtype) -> "DeviceTensor":
        """Borrows caller-owned device memory (e.g. torch `tensor.data_ptr()`)."""
        h = ctypes.c_void_p()
        N.check(self.lib.b2m_tensor_wrap(self.handle, ctypes.c_void_p(device_ptr), b2m_dtype(dtype),
                                         _shape_arr(shape), len(shape), ctypes.byref(h)))
        return DeviceTensor(self, h)

    # -- weights -----------------------------------------------------------
    def prepack_f32(self, b, trans: bool = False) -> "PackedWeight":
        b = np.ascontiguousarray(b, np.float32)
        if b.ndim != 2:
            raise N.ArgumentError("Gemm prepack: B must be 2-D")
        h = ctypes.c_void_p()
        N.check(self.lib.b2m_weight_prepack_f32(self.handle, b.ctypes.data_as(ctypes.c_void_p), b.shape[0],
                                                b.shape[1], 1 if trans else 0, ctypes.byref(h)))
        return PackedWeight(self, h, "f32")

    def prepack_i8(self, b) -> "PackedWeight":
        b = np.ascontiguousarray(b)
        if b.ndim != 2 or b.dtype not in (np.uint8, np.int8):
            raise N.ArgumentError("MatMulInteger prepack: B must be a 2-D uint8/int8 matrix")
        h = ctypes.c_void_p()
        N.check(self.lib.b2m_weight_prepack_i8(self.handle, b.ctypes.data_as(ctypes.c_void_p), b2m_dtype(b.dtype),
                                               b.shape[0], b.shape[1], ctypes.byref(h)))
        return PackedWeight(self, h, "i8")

    def prepack_conv(self, w) -> "PackedWeight":
        """Conv / ConvInteger / QLinearConv weight [M][C/group][kernel...]
        (float32, uint8 or int8) packed as the GEMM operand; the result keeps
        the ONNX weight shape in `.shape`."""
        w = np.ascontiguousarray(w)
        if w.ndim < 3 or w.dtype not in (np.float32, np.uint8, np.int8):
            raise N.ArgumentError("Conv prepack: weight must be [M][C/group][kernel...] float32, uint8 or int8")
        m = int(w.shape[0])
        k = int(np.prod(w.shape[1:]))
        h = ctypes.c_void_p()
        N.check(self.lib.b2m_weight_prepack_conv(self.handle, w.ctypes.data_as(ctypes.c_void_p), b2m_dtype(w.dtype),
                                                 m, k, ctypes.byref(h)))
        pw = PackedWeight(self, h, "f32" if w.dtype == np.float32 else "i8")
        pw.shape = tuple(int(d) for d in w.shape)
        return pw

    def prepack_nbits(self, b_q, scales, zero_points, k: int, n: int, bits: int, block_size: int) -> "PackedWeight":
        bq = np.ascontiguousarray(b_q, np.uint8)
        sc = np.ascontiguousarray(scales, np.float32)
        zp_ptr, zp_dt, zp = None, 0, None
        if zero_points is not None:
            zp = np.ascontiguousarray(zero_points)
            zp_dt = N.B2M_UINT8 if zp.dtype == np.uint8 else N.B2M_FLOAT
            if zp_dt == N.B2M_FLOAT:
                zp = np.ascontiguousarray(zp, np.float32)
            zp_ptr = zp.ctypes.data_as(ctypes.c_void_p)
        h = ctypes.c_void_p()
        N.check(self.lib.b2m_weight_prepack_nbits(self.handle, bq.ctypes.data_as(ctypes.c_void_p),
                                                  sc.ctypes.data_as(ctypes.c_void_p), zp_ptr, zp_dt, int(k), int(n),
                                                  int(bits), int(block_size), ctypes.byref(h)))
        return PackedWeight(self, h, "nbits")

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class DeviceTensor:
    """A device-resident tensor handle (b2m_tensor)."""

    def __init__(self, ctx: Context, handle):
        self.ctx = ctx
        self.handle = handle

    def _info(self):
        dt, rk = ctypes.c_int32(), ctypes.c_int32()
        shp = (ctypes.c_int64 * N.MAX_RANK)()
        ptr = ctypes.c_void_p()
        N.check(self.ctx.lib.b2m_tensor_info(self.handle, ctypes.byref(dt), ctypes.byref(rk), shp, ctypes.byref(ptr)))
        return dt.value, [int(shp[i]) for i in range(rk.value)], ptr.value

    @property
    def shape(self):
        return self._info()[1]

    @property
    def dtype(self):
        return np_dtype(self._info()[0])

    @property
    def data_ptr(self) -> int:
        return self._info()[2] or 0

    @property
    def rank(self):
        return len(self.shape)

    def numpy(self) -> np.ndarray:
        code, shape, _ = self._info()
        out = np.empty(shape, np_dtype(code))
        N.check(self.ctx.lib.b2m_tensor_download(self.ctx.handle, self.handle, out.ctypes.data_as(ctypes.c_void_p),
                                                 out.nbytes))
        return out

    def free(self):
        if self.handle:
            N.check(self.ctx.lib.b2m_tensor_free(self.handle))
            self.handle = None

    def __del__(self):
        try:
            if self.handle and self.ctx.handle:
                self.ctx.lib.b2m_tensor_free(self.handle)
                self.handle = None
        except Exception:
            pass


class PackedWeight:
    """A prepacked initializer (b2m_weight)."""

    def __init__(self, ctx: Context, handle, kind: str):
        self.ctx = ctx
        self.handle = handle
        self.kind = kind
        self.shape = None  # ONNX weight shape of a convolution weight

    @property
    def kn(self):
        k, n = ctypes.c_int64(), ctypes.c_int64()
        N.check(self.ctx.lib.b2m_weight_info(self.handle, ctypes.byref(k), ctypes.byref(n)))
        return int(k.value), int(n.value)

    def set_next(self, nxt: "PackedWeight | None"):
        """Declares the MatMulNBits weight of the call that follows this
        weight's calls (b2m_weight_set_next): their kernels prefetch it into
        L2. A hint; None clears it."""
        N.check(self.ctx.lib.b2m_weight_set_next(self.handle, None if nxt is None else nxt.handle))

    def free(self):
        if self.handle:
            N.check(self.ctx.lib.b2m_weight_free(self.handle))
            self.handle = None

    def __del__(self):
        try:
            if self.handle and self.ctx.handle:
                self.ctx.lib.b2m_weight_free(self.handle)
                self.handle = None
        except Exception:
            pass


@contextlib.contextmanager
def torch_stream_scope(ctx: Context, torch, own):
    """Orders the enclosed library calls with torch's current stream.

    b2m_set_stream(NULL) selects the context's own stream, so the legacy default
    stream (handle 0) cannot be passed through; when it is current, the work
    runs on `own` (a torch stream of the same device), which first waits for the
    caller's stream and which the caller's stream waits for on exit."""
    cur = torch.cuda.current_stream()
    if cur.cuda_stream != 0:
        ctx.set_stream(cur.cuda_stream)
        yield cur
        return
    own.wait_stream(cur)
    try:
        with torch.cuda.stream(own):
            ctx.set_stream(own.cuda_stream)
            yield own
    finally:
        cur.wait_stream(own)
