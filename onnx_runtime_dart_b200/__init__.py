"""B200 (sm_100a) backend for the MatMul-family operators of onnx_runtime_dart.

The compute lives in libb200mm.so (CUDA kernels behind the C ABI of
include/b2m.h); this package is the host-side mirror of the reference's
operator interface over that ABI. See `ops` for the operators and `dispatch`
for the executor hook.
"""
from ._native import (ArgumentError, B2mError, DeviceTimeoutError, NoDeviceError, OnnxCancelledException,
                      OnnxMemoryLimitException, UnsupportedError)
from .ops import (MODE_EXACT, MODE_FAST, MODE_PRECISE, opDynamicQuantizeLinear, opGemm, opMatMul, opMatMulInteger,
                  opMatMulNBits, opQLinearMatMul, prepack_nbits, validate_nbits)
from .runtime import Context, DeviceTensor, PackedWeight

__all__ = [
    "ArgumentError", "B2mError", "DeviceTimeoutError", "NoDeviceError", "OnnxCancelledException",
    "OnnxMemoryLimitException", "UnsupportedError", "MODE_EXACT", "MODE_FAST", "MODE_PRECISE",
    "opDynamicQuantizeLinear", "opGemm", "opMatMul", "opMatMulInteger", "opMatMulNBits", "opQLinearMatMul",
    "prepack_nbits", "validate_nbits", "Context", "DeviceTensor", "PackedWeight",
]
