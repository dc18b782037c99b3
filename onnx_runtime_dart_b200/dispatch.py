"""Operator-dispatch hook: the MatMul-family cases of the reference's
OnnxGraphExecutor._dispatch (lib/src/onnx_graph.dart:1549), routed to the GPU.

`GpuDispatch.dispatch(op_type, input_names, values, attrs)` follows the
reference's cases line for line:
  'MatMul'        onnx_graph.dart:2154-2155
  'Gemm'          onnx_graph.dart:2156-2173  (transB initializer prepacked once)
  'MatMulInteger' onnx_graph.dart:2880-2888
  'QLinearMatMul' onnx_graph.dart:2902-2917  (lo/hi from y_zero_point's elem type)
  'MatMulNBits'   onnx_graph.dart:2918-2934  (g_idx rejected)
  'Conv'          onnx_graph.dart:2436-2490  (kernel_shape checked against the weight)
  'ConvInteger'   onnx_graph.dart:2889-2901
  'QLinearConv'   onnx_graph.dart:2935-2956  (lo/hi from y_zero_point's elem type)
  'ConvTranspose' onnx_graph.dart:2491-2515  (kernel_shape checked against the weight)
Initializer weights are prepacked on first use and cached by initializer name
(the reference's `_prepackedGemmB`, onnx_graph.dart:102-105); the graph itself
is unchanged. Ops outside the family return None, leaving the reference's own
op to run.
"""
from __future__ import annotations

import numpy as np

from . import _native as N
from . import ops
from .runtime import Context, DeviceTensor


class GpuDispatch:
    HANDLED = ("MatMul", "Gemm", "MatMulInteger", "QLinearMatMul", "MatMulNBits", "Conv", "ConvInteger",
               "QLinearConv", "ConvTranspose")

    def __init__(self, ctx: Context, initializers: dict, initializer_elem_types: dict | None = None,
                 f32_mode: int = ops.MODE_EXACT, nbits_mode: int = ops.MODE_FAST):
        self.ctx = ctx
        self.initializers = initializers
        self.elem_types = initializer_elem_types or {}
        self.f32_mode = f32_mode
        self.nbits_mode = nbits_mode
        self._packed = {}

    def _is_init(self, name):
        return bool(name) and name in self.initializers

    def _packed_for(self, key, make):
        w = self._packed.get(key)
        if w is None:
            w = make()
            self._packed[key] = w
        return w

    def dispatch(self, op_type: str, input_names: list, values: list, attrs: dict, outputs: list | None = None):
        """Runs one node; returns its outputs (device tensors), or None for ops
        outside the family. `outputs` optionally names caller-owned device
        tensors the MatMulNBits output is written into (so a chain can keep
        fixed buffers, e.g. inside a captured CUDA graph)."""
        if op_type not in self.HANDLED:
            return None

        def need(i):
            v = values[i] if i < len(values) else None
            if v is None:
                raise N.ArgumentError(f"{op_type}: missing required input {i}")
            return v

        def opt(i):
            return values[i] if i < len(values) else None

        ctx = self.ctx
        if op_type == "MatMul":
            b = need(1)
            if self._is_init(input_names[1]) and np.ndim(b) == 2 and not isinstance(b, DeviceTensor):
                b = self._packed_for(("f32", input_names[1]), lambda: ctx.prepack_f32(np.asarray(b)))
            return [ops.opMatMul(need(0), b, mode=self.f32_mode, ctx=ctx)]
        if op_type == "Gemm":
            b = need(1)
            trans_b = int(attrs.get("transB", 0)) != 0
            if self._is_init(input_names[1]) and not isinstance(b, DeviceTensor):
                # prepack = the one-time transpose of the reference (:2159-2161)
                b = self._packed_for(("gemm", input_names[1], trans_b),
                                     lambda: ctx.prepack_f32(np.asarray(b), trans=trans_b))
                trans_b = False
            return [ops.opGemm(need(0), b, opt(2), alpha=float(attrs.get("alpha", 1.0)),
                               beta=float(attrs.get("beta", 1.0)), transA=int(attrs.get("transA", 0)) != 0,
                               transB=trans_b, mode=self.f32_mode, ctx=ctx)]
        if op_type == "MatMulInteger":
            b = need(1)
            if self._is_init(input_names[1]) and np.ndim(b) == 2 and not isinstance(b, DeviceTensor):
                b = self._packed_for(("i8", input_names[1]), lambda: ctx.prepack_i8(np.asarray(b)))
            return [ops.opMatMulInteger(need(0), b, opt(2), opt(3), ctx=ctx)]
        if op_type == "QLinearMatMul":
            int8 = self.elem_types.get(input_names[7] if len(input_names) > 7 else "", 0) == 3
            b = need(3)
            if self._is_init(input_names[3]) and np.ndim(b) == 2 and not isinstance(b, DeviceTensor):
                b = self._packed_for(("i8", input_names[3]), lambda: ctx.prepack_i8(np.asarray(b)))
            return [ops.opQLinearMatMul(need(0), need(1), opt(2), b, need(4), opt(5), need(6), opt(7),
                                        lo=-128 if int8 else 0, hi=127 if int8 else 255, ctx=ctx)]
        if op_type in ("Conv", "ConvInteger", "QLinearConv"):
            return [self._conv(op_type, input_names, need, opt, attrs)]
        if op_type == "ConvTranspose":
            w = need(1)
            declared = attrs.get("kernel_shape")
            kernel = [int(v) for v in (w.shape if hasattr(w, "shape") else np.shape(w))[2:]]
            if declared is not None and [int(v) for v in declared] != kernel:
                raise N.StateError(f"ConvTranspose kernel_shape {list(declared)} does not match weight shape "
                                   f"{kernel}.")
            if self._is_init(input_names[1]) and not isinstance(w, DeviceTensor):
                w = self._packed_for(("convT", input_names[1]), lambda: ctx.upload(np.asarray(w, np.float32)))
            return [ops.opConvTranspose(need(0), w, opt(2), strides=attrs.get("strides"), pads=attrs.get("pads"),
                                        dilations=attrs.get("dilations"), outputPadding=attrs.get("output_padding"),
                                        outputShape=attrs.get("output_shape"), group=int(attrs.get("group", 1)),
                                        ctx=ctx)]
        # MatMulNBits
        if len(input_names) > 4 and input_names[4]:
            raise N.UnsupportedError("MatMulNBits: g_idx input not supported")
        k, n = int(attrs["K"]), int(attrs["N"])
        bits = int(attrs.get("bits", 4))
        block = int(attrs["block_size"])
        zp = opt(3)
        bias = opt(5)
        a = need(0)
        ops.validate_nbits(list(a.shape), a.dtype, np.asarray(need(1)), np.asarray(need(2)),
                           None if zp is None else np.asarray(zp),
                           None if bias is None or isinstance(bias, DeviceTensor) else np.asarray(bias),
                           k, n, bits, block)
        key = ("nbits", input_names[1], input_names[2], input_names[3] if len(input_names) > 3 else "")
        if self._is_init(input_names[1]):
            w = self._packed_for(key, lambda: ops.prepack_nbits(ctx, need(1), need(2), zp, k=k, n=n, bits=bits,
                                                                blockSize=block))
        else:
            w = ops.prepack_nbits(ctx, need(1), need(2), zp, k=k, n=n, bits=bits, blockSize=block)
        return [ops.opMatMulNBits(a, w, k=k, n=n, bits=bits, blockSize=block, bias=bias, mode=self.nbits_mode,
                                  ctx=ctx, out=outputs[0] if outputs else None)]

    def _conv(self, op_type, input_names, need, opt, attrs):
        ctx = self.ctx
        wi = 3 if op_type == "QLinearConv" else 1
        w = need(wi)
        if op_type == "Conv":
            declared = attrs.get("kernel_shape")
            kernel = [int(v) for v in (w.shape if hasattr(w, "shape") else np.shape(w))[2:]]
            if declared is not None and [int(v) for v in declared] != kernel:
                raise N.StateError(f"Conv kernel_shape {list(declared)} does not match weight shape {kernel}.")
        if self._is_init(input_names[wi]) and not isinstance(w, DeviceTensor):
            w = self._packed_for(("conv", input_names[wi]), lambda: ctx.prepack_conv(np.asarray(w)))
        spatial = dict(strides=attrs.get("strides"), pads=attrs.get("pads"), dilations=attrs.get("dilations"),
                       group=int(attrs.get("group", 1)))
        if op_type == "Conv":
            return ops.opConv(need(0), w, opt(2), autoPad=attrs.get("auto_pad", "NOTSET") or "NOTSET",
                              mode=self.f32_mode, ctx=ctx, **spatial)
        if op_type == "ConvInteger":
            return ops.opConvInteger(need(0), w, opt(2), opt(3), ctx=ctx, **spatial)
        int8 = self.elem_types.get(input_names[7] if len(input_names) > 7 else "", 0) == 3
        return ops.opQLinearConv(need(0), need(1), opt(2), w, need(4), opt(5), need(6), opt(7), opt(8),
                                 lo=-128 if int8 else 0, hi=127 if int8 else 255, ctx=ctx, **spatial)
