"""ctypes binding of libb200mm.so (include/b2m.h).

This is the Python counterpart of the dart:ffi binding a Dart caller would
use: it opens the library, declares the entry points, and turns status codes into the exception classes the reference
throws (ArgumentError, UnsupportedError, OnnxMemoryLimitException,
OnnxCancelledException — lib/src/onnx_qlinear_ops.dart:127-165,
lib/src/execution_control.dart). Library discovery follows the reference's
native-library lookup order (lib/src/ort/ort_backend.dart:1221-1277):
explicit path, then the B2M_LIBRARY environment variable, then the copy built
next to this file.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))

B2M_OK = 0
B2M_ERR_INVALID_ARGUMENT = 1
B2M_ERR_UNSUPPORTED = 2
B2M_ERR_OUT_OF_MEMORY = 3
B2M_ERR_CUDA = 4
B2M_ERR_TIMEOUT = 5
B2M_ERR_CANCELLED = 6
B2M_ERR_NO_DEVICE = 7

B2M_FLOAT = 1
B2M_UINT8 = 2
B2M_INT8 = 3
B2M_INT32 = 6
B2M_INT64 = 7
B2M_FLOAT16 = 10

MODE_EXACT = 0
MODE_FAST = 1
MODE_PRECISE = 2  # MatMulNBits: bf16-split products on exactly dequantized weights
ROUTE_GEMV, ROUTE_TC_F16, ROUTE_OTHER = 0, 1, 2  # b2m_matmul_nbits_route

MAX_RANK = 8
NOALLOC_SCRATCH_BYTES = 8 << 20


class B2mError(RuntimeError):
    """Base class of errors raised through the C ABI."""

    status = B2M_ERR_CUDA


class ArgumentError(B2mError, ValueError):
    """Dart ArgumentError: invalid shapes or values."""

    status = B2M_ERR_INVALID_ARGUMENT


class StateError(B2mError):
    """Dart StateError: the executor's node-level consistency checks (e.g.
    Conv's kernel_shape against the weight, onnx_graph.dart:2440-2446)."""

    status = B2M_ERR_INVALID_ARGUMENT


class UnsupportedError(B2mError, NotImplementedError):
    """Dart UnsupportedError: a valid but unsupported feature."""

    status = B2M_ERR_UNSUPPORTED


class OnnxMemoryLimitException(B2mError, MemoryError):
    """Device allocation failed or the context's byte budget was exceeded."""

    status = B2M_ERR_OUT_OF_MEMORY


class OnnxCancelledException(B2mError):
    """The context's cancel flag was set (OnnxExecutionControl.checkpoint)."""

    status = B2M_ERR_CANCELLED


class DeviceTimeoutError(B2mError):
    """A bounded device-side wait gave up."""

    status = B2M_ERR_TIMEOUT


class NoDeviceError(B2mError):
    status = B2M_ERR_NO_DEVICE


_ERRORS = {c.status: c for c in (ArgumentError, UnsupportedError, OnnxMemoryLimitException,
                                 OnnxCancelledException, DeviceTimeoutError, NoDeviceError)}

_c_ctx = ctypes.c_void_p
_c_tensor = ctypes.c_void_p
_c_weight = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float
_vp = ctypes.c_void_p
_i64p = ctypes.POINTER(ctypes.c_int64)
_i32p = ctypes.POINTER(ctypes.c_int32)

# name -> (restype, argtypes); the full export list of include/b2m.h.
SIGNATURES = {
    "b2m_abi_version": (_i32, []),
    "b2m_last_error": (ctypes.c_char_p, []),
    "b2m_device_count": (_i32, [_i32p]),
    "b2m_init": (_i32, [_i32, ctypes.POINTER(_c_ctx)]),
    "b2m_shutdown": (_i32, [_c_ctx]),
    "b2m_set_stream": (_i32, [_c_ctx, _vp]),
    "b2m_synchronize": (_i32, [_c_ctx]),
    "b2m_set_cancel_flag": (_i32, [_c_ctx, _i32p]),
    "b2m_set_byte_budget": (_i32, [_c_ctx, _i64]),
    "b2m_set_attention_mode": (_i32, [_c_ctx, _i32]),
    "b2m_weight_set_next": (_i32, [_c_weight, _c_weight]),
    "b2m_rmsnorm_head_rows_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_double]),
    "b2m_enable_timing": (_i32, [_c_ctx, _i32]),
    "b2m_last_kernel_ms": (_i32, [_c_ctx, ctypes.POINTER(_f32)]),
    "b2m_tensor_alloc": (_i32, [_c_ctx, _i32, _i64p, _i32, ctypes.POINTER(_c_tensor)]),
    "b2m_tensor_wrap": (_i32, [_c_ctx, _vp, _i32, _i64p, _i32, ctypes.POINTER(_c_tensor)]),
    "b2m_tensor_upload": (_i32, [_c_ctx, _c_tensor, _vp, _i64]),
    "b2m_tensor_download": (_i32, [_c_ctx, _c_tensor, _vp, _i64]),
    "b2m_tensor_free": (_i32, [_c_tensor]),
    "b2m_host_alloc": (_i32, [_c_ctx, _i64, ctypes.POINTER(_vp)]),
    "b2m_host_free": (_i32, [_c_ctx, _vp]),
    "b2m_tensor_info": (_i32, [_c_tensor, _i32p, _i32p, _i64p, ctypes.POINTER(_vp)]),
    "b2m_weight_prepack_f32": (_i32, [_c_ctx, _vp, _i64, _i64, _i32, ctypes.POINTER(_c_weight)]),
    "b2m_weight_prepack_i8": (_i32, [_c_ctx, _vp, _i32, _i64, _i64, ctypes.POINTER(_c_weight)]),
    "b2m_weight_prepack_nbits": (_i32, [_c_ctx, _vp, _vp, _vp, _i32, _i64, _i64, _i32, _i32,
                                        ctypes.POINTER(_c_weight)]),
    "b2m_weight_free": (_i32, [_c_weight]),
    "b2m_weight_prepack_conv": (_i32, [_c_ctx, _vp, _i32, _i64, _i64, ctypes.POINTER(_c_weight)]),
    "b2m_conv_transpose_f32": (_i32, [_c_ctx, _c_tensor, _c_tensor, _c_tensor, _vp, _vp, _vp, _vp, _vp, _i32,
                                      ctypes.POINTER(_c_tensor)]),
    "b2m_conv_f32": (_i32, [_c_ctx, _c_tensor, _c_weight, _c_tensor, _vp, _vp, _vp, _vp, _i32, _i32, _i32,
                            ctypes.POINTER(_c_tensor)]),
    "b2m_conv_integer": (_i32, [_c_ctx, _c_tensor, _c_tensor, _c_weight, _c_tensor, _vp, _vp, _vp, _vp, _i32,
                                ctypes.POINTER(_c_tensor)]),
    "b2m_qlinear_conv": (_i32, [_c_ctx, _c_tensor, _f32, _c_tensor, _c_weight, _c_tensor, _c_tensor, _f32, _i32,
                                _c_tensor, _vp, _vp, _vp, _vp, _i32, _i32, _i32, ctypes.POINTER(_c_tensor)]),
    "b2m_weight_info": (_i32, [_c_weight, _i64p, _i64p]),
    "b2m_matmul_f32": (_i32, [_c_ctx, _c_tensor, _c_tensor, _c_weight, _i32, ctypes.POINTER(_c_tensor)]),
    "b2m_gemm_f32": (_i32, [_c_ctx, _c_tensor, _c_tensor, _c_weight, _c_tensor, _f32, _f32, _i32, _i32, _i32,
                            ctypes.POINTER(_c_tensor)]),
    "b2m_matmul_integer": (_i32, [_c_ctx, _c_tensor, _c_tensor, _c_weight, _c_tensor, _c_tensor,
                                  ctypes.POINTER(_c_tensor)]),
    "b2m_qlinear_matmul": (_i32, [_c_ctx, _c_tensor, _f32, _c_tensor, _c_tensor, _c_weight, _f32, _c_tensor,
                                  _f32, _i32, _i32, _i32, ctypes.POINTER(_c_tensor)]),
    "b2m_matmul_nbits": (_i32, [_c_ctx, _c_tensor, _c_weight, _c_tensor, _i32, ctypes.POINTER(_c_tensor)]),
    "b2m_matmul_nbits_host": (_i32, [_c_ctx, _vp, _i64, _c_weight, _vp, _i32, _vp]),
    "b2m_matmul_nbits_dev": (_i32, [_c_ctx, _vp, _i64, _c_weight, _vp, _i32, _vp]),
    "b2m_matmul_nbits_noalloc": (_i32, [_c_weight, _vp, _i64, _vp, _vp, _vp]),
    "b2m_rmsnorm_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_double]),
    "b2m_rmsnorm_heads_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.c_double]),
    "b2m_layernorm_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_double]),
    "b2m_silu_mul_dev": (_i32, [_c_ctx, _vp, _vp, _i64, _i64, _vp, _i64, _i64]),
    "b2m_silu_mul_f16_dev": (_i32, [_c_ctx, _vp, _vp, _i64, _i64, _vp, _vp, _i64, _i64]),
    "b2m_layernorm_split_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_double]),
    "b2m_gelu_split_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _i64, _i64]),
    "b2m_gemm_f32_split_dev": (_i32, [_c_ctx, _vp, _i64, _c_weight, _vp, _vp]),
    "b2m_rmsnorm_f16_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_double]),
    "b2m_matmul_nbits_route": (_i32, [_c_ctx, _c_weight, _i64, _i32, ctypes.POINTER(_i32)]),
    "b2m_matmul_nbits_f16_dev": (_i32, [_c_ctx, _vp, _i64, _c_weight, _vp, _vp]),
    "b2m_matmul_nbits_swiglu_dev": (_i32, [_c_ctx, _vp, _vp, _i64, _c_weight, _i32, _vp, _vp]),
    "b2m_gelu_dev": (_i32, [_c_ctx, _vp, _vp, _i64]),
    "b2m_add_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _i64, _i64, _i32]),
    "b2m_gather_rows_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _i64, _i64, _i64]),
    "b2m_argmax_dev": (_i32, [_c_ctx, _vp, _vp, _i64, _i64]),
    "b2m_gqa_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _i32,
                           _i32, _i32, _i32, _i32, _i32, _f32]),
    "b2m_gqa_f16_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp, _vp,
                               _i32, _i32, _i32, _i32, _i32, _i32, _f32]),
    "b2m_gqa_qknorm_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _i64, _i64, _vp, ctypes.c_double, _vp, _vp, _vp, _vp, _vp,
                                  _i32, _i32, _i32, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _f32]),
    "b2m_mha_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _i32, _i32, _i32, _i32,
                           _i32, _i32, _f32, _i32]),
    "b2m_mha_split_dev": (_i32, [_c_ctx, _vp, _vp, _vp, _i64, _i64, _vp, _i64, _i64, _i64, _vp, _vp, _i32, _i32,
                                 _i32, _i32, _i32, _i32, _f32, _i32]),
    "b2m_dynamic_quantize_linear_dev": (_i32, [_c_ctx, _vp, _i64, _vp, _vp, _vp]),
    "b2m_rotary_dev": (_i32, [_c_ctx, _vp, _i64, _vp, _i32, _vp, _vp, _i32, _i32, _vp, _i64, _i32, _i32, _i32,
                              _i32, _i32, _i32]),
    "b2m_advance_positions_dev": (_i32, [_c_ctx, _vp, _i32, _i32]),
    "b2m_weight_export": (_i32, [_c_weight, _vp, ctypes.c_size_t, ctypes.POINTER(ctypes.c_size_t)]),
    "b2m_weight_import": (_i32, [_c_ctx, _vp, ctypes.c_size_t, ctypes.POINTER(_c_weight)]),
}

_lib = None


def library_path(explicit: str | None = None) -> str:
    for cand in (explicit, os.environ.get("B2M_LIBRARY"), os.path.join(HERE, "libb200mm.so")):
        if cand and os.path.exists(cand):
            return cand
    raise OSError("libb200mm.so not found: build it with `python -m onnx_runtime_dart_b200.build` "
                  "or point B2M_LIBRARY at it")


def load(explicit: str | None = None):
    """Opens the library once and declares every entry point."""
    global _lib
    if _lib is not None:
        return _lib
    lib = ctypes.CDLL(library_path(explicit))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status: int) -> None:
    """Raises the exception class matching a non-zero b2m_status."""
    if status == B2M_OK:
        return
    msg = load().b2m_last_error().decode(errors="replace")
    raise _ERRORS.get(status, B2mError)(msg or f"b2m status {status}")
