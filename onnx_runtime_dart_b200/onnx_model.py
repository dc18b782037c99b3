"""Load-time prepack: reads an ONNX model's graph and initializers (including
external data) and packs every MatMul-family weight for the device once, at
session load, optionally through an on-disk cache of packed layouts.

Reference: the protobuf loader's tensor decoding (tensorFromProto,
lib/src/onnx_proto_loader.dart:171-299: float / float16 / double / int8 /
uint8 / int32 / int64 / int4 / uint4 / bool, inline typed fields or
raw_data, external data by location / offset / length resolved next to the
model file, :100-124) and the executor's per-initializer prepack cache
(`_prepackedGemmB`, lib/src/onnx_graph.dart:102-105, 2156-2173). The
reference packs lazily on first use; here `prepack_session` packs every
weight the MatMul-family dispatch will ask for before the first run, keyed
exactly as `dispatch.GpuDispatch` looks them up.

The protobuf wire format is read directly (no onnx package): field numbers of
the ONNX schema, ModelProto.graph = 7; GraphProto node = 1, initializer = 5,
input = 11, output = 12; NodeProto input = 1, output = 2, op_type = 4,
attribute = 5, domain = 7; AttributeProto name = 1, f = 2, i = 3, s = 4,
t = 5, floats = 7, ints = 8; TensorProto dims = 1, data_type = 2,
float_data = 4, int32_data = 5, int64_data = 7, name = 8, raw_data = 9,
double_data = 10, external_data = 13, data_location = 14.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import struct
from dataclasses import dataclass, field

import numpy as np

from . import _native as N

# TensorProto.DataType values the loader decodes.
FLOAT, UINT8, INT8, INT32, INT64, BOOL, FLOAT16, DOUBLE, UINT4, INT4 = 1, 2, 3, 6, 7, 9, 10, 11, 21, 22


def _varint(buf, pos):
    out = shift = 0
    while True:
        b = buf[pos]
        pos += 1
        out |= (b & 0x7F) << shift
        if not b & 0x80:
            return out, pos
        shift += 7


def _fields(buf):
    """(field number, wire type, value) of one message; value is an int for
    varints, bytes for fixed / length-delimited fields."""
    pos, n = 0, len(buf)
    while pos < n:
        key, pos = _varint(buf, pos)
        fn, wt = key >> 3, key & 7
        if wt == 0:
            v, pos = _varint(buf, pos)
        elif wt == 1:
            v, pos = buf[pos:pos + 8], pos + 8
        elif wt == 2:
            ln, pos = _varint(buf, pos)
            v, pos = buf[pos:pos + ln], pos + ln
        elif wt == 5:
            v, pos = buf[pos:pos + 4], pos + 4
        else:
            raise ValueError(f"ONNX protobuf: unsupported wire type {wt}")
        yield fn, wt, v


def _s64(v):
    return v - (1 << 64) if v >= 1 << 63 else v


def _ints(v, wt):
    if wt == 0:
        return [_s64(v)]
    out, pos = [], 0
    while pos < len(v):
        x, pos = _varint(v, pos)
        out.append(_s64(x))
    return out


def _floats(v, wt, fmt="f"):
    size = struct.calcsize(fmt)
    if wt == 2:
        return list(struct.unpack(f"<{len(v) // size}{fmt}", v))
    return [struct.unpack(f"<{fmt}", v)[0]]


@dataclass
class TensorInfo:
    name: str
    data_type: int
    dims: list
    array: np.ndarray


@dataclass
class Node:
    op_type: str
    domain: str
    inputs: list
    outputs: list
    attrs: dict = field(default_factory=dict)


@dataclass
class OnnxModel:
    path: str
    nodes: list
    initializers: dict          # name -> numpy array
    elem_types: dict            # name -> TensorProto.DataType of each initializer
    inputs: list
    outputs: list


def _element_count(dims, name):
    n = 1
    for d in dims:
        if d < 0:
            raise ValueError(f'Tensor "{name}" has a negative dimension {d}')
        n *= d
    return n


def decode_tensor(buf, model_dir: str | None = None) -> TensorInfo:
    """TensorProto bytes -> numpy, following tensorFromProto's rules (float16
    and double widened / narrowed to float32, int32 carried as int64, int4 /
    uint4 unpacked low nibble first, bool as int64 0 / 1)."""
    dims, dt, name, raw = [], 0, "", None
    f32, i32, i64, f64 = [], [], [], []
    ext, location = {}, 0
    for fn, wt, v in _fields(buf):
        if fn == 1:
            dims += _ints(v, wt)
        elif fn == 2:
            dt = v
        elif fn == 4:
            f32 += _floats(v, wt)
        elif fn == 5:
            i32 += _ints(v, wt)
        elif fn == 7:
            i64 += _ints(v, wt)
        elif fn == 8:
            name = bytes(v).decode()
        elif fn == 9:
            raw = bytes(v)
        elif fn == 10:
            f64 += _floats(v, wt, "d")
        elif fn == 13:
            kv = {f: bytes(x).decode() for f, _, x in _fields(v)}
            ext[kv.get(1, "")] = kv.get(2, "")
        elif fn == 14:
            location = v
    n = _element_count(dims, name)
    width = {FLOAT: 4, UINT8: 1, INT8: 1, INT32: 4, INT64: 8, BOOL: 1, FLOAT16: 2, DOUBLE: 8}.get(dt)

    def raw_bytes(expect):
        if location == 1:
            if model_dir is None:
                raise RuntimeError(f'"{name}" stores its weights externally: load the model from its file so the '
                                   "companion data file is found")
            offset = int(ext.get("offset", "0") or 0)
            length = int(ext.get("length", "0") or 0) or expect
            with open(os.path.join(model_dir, ext.get("location", "")), "rb") as f:
                f.seek(offset)
                return f.read(length)
        return raw if raw is not None else b""

    def need_raw(have, elem):
        if n > have // elem:
            raise ValueError(f'Tensor "{name}" raw_data too short: {have} bytes for {n} elements of {elem} bytes')

    def need_inline(have):
        if have != n:
            raise ValueError(f'Tensor "{name}" inline data length {have} does not match shape product {n}')

    if dt == FLOAT and f32:
        need_inline(len(f32))
        arr = np.array(f32, np.float32)
    elif dt == INT64 and i64:
        need_inline(len(i64))
        arr = np.array(i64, np.int64)
    elif dt == INT32 and i32:
        need_inline(len(i32))
        arr = np.array(i32, np.int64)
    elif dt == DOUBLE and f64:
        need_inline(len(f64))
        arr = np.array(f64, np.float64).astype(np.float32)
    elif dt in (UINT8, INT8) and i32:
        need_inline(len(i32))
        arr = np.array(i32, np.int64).astype(np.int8 if dt == INT8 else np.uint8)
    elif dt in (UINT4, INT4):
        b = np.frombuffer(raw_bytes((n + 1) // 2), np.uint8)
        need_raw(len(b) * 2, 1)
        nib = np.empty(len(b) * 2, np.uint8)
        nib[0::2], nib[1::2] = b & 0xF, b >> 4
        nib = nib[:n]
        arr = (np.where(nib > 7, nib.astype(np.int16) - 16, nib).astype(np.int8) if dt == INT4 else nib)
    elif width is not None:
        b = raw_bytes(n * width)
        need_raw(len(b), width)
        np_dt = {FLOAT: "<f4", UINT8: "u1", INT8: "i1", INT32: "<i4", INT64: "<i8", BOOL: "u1", FLOAT16: "<f2",
                 DOUBLE: "<f8"}[dt]
        arr = np.frombuffer(b, np_dt, count=n)
        if dt in (FLOAT16, DOUBLE):
            arr = arr.astype(np.float32)
        elif dt in (INT32, BOOL):
            arr = (arr != 0).astype(np.int64) if dt == BOOL else arr.astype(np.int64)
        else:
            arr = arr.copy()
    else:
        raise N.UnsupportedError(f'Unsupported ONNX TensorProto dataType {dt} for "{name}"')
    return TensorInfo(name, dt, dims, arr.reshape(dims))


def _attribute(buf, model_dir):
    name, val = "", None
    for fn, wt, v in _fields(buf):
        if fn == 1:
            name = bytes(v).decode()
        elif fn == 2:
            val = struct.unpack("<f", v)[0]
        elif fn == 3:
            val = _s64(v)
        elif fn == 4:
            val = bytes(v).decode(errors="replace")
        elif fn == 5:
            val = decode_tensor(v, model_dir).array
        elif fn == 7:
            val = (val or []) + _floats(v, wt)
        elif fn == 8:
            val = (val or []) + _ints(v, wt)
    return name, val


def load_model(path: str) -> OnnxModel:
    """Reads the graph's nodes, inputs, outputs and initializers."""
    model_dir = os.path.dirname(os.path.abspath(path))
    with open(path, "rb") as f:
        buf = memoryview(f.read())
    graph = next((v for fn, _, v in _fields(buf) if fn == 7), None)
    if graph is None:
        raise ValueError(f"{path}: no graph in the model")
    nodes, inits, types, ins, outs = [], {}, {}, [], []
    for fn, _, v in _fields(graph):
        if fn == 1:
            nd = Node("", "", [], [])
            for f2, _, x in _fields(v):
                if f2 == 1:
                    nd.inputs.append(bytes(x).decode())
                elif f2 == 2:
                    nd.outputs.append(bytes(x).decode())
                elif f2 == 4:
                    nd.op_type = bytes(x).decode()
                elif f2 == 5:
                    k, val = _attribute(x, model_dir)
                    nd.attrs[k] = val
                elif f2 == 7:
                    nd.domain = bytes(x).decode()
            nodes.append(nd)
        elif fn == 5:
            t = decode_tensor(v, model_dir)
            inits[t.name] = t.array
            types[t.name] = t.data_type
        elif fn in (11, 12):
            nm = next((bytes(x).decode() for f2, _, x in _fields(v) if f2 == 1), "")
            (ins if fn == 11 else outs).append(nm)
    return OnnxModel(path, nodes, inits, types, ins, outs)


# ---------------------------------------------------------------------------
# Load-time prepack with an on-disk cache of packed layouts
# ---------------------------------------------------------------------------

def _cache_key(kind: str, parts, arrays) -> str:
    h = hashlib.sha256()
    h.update(kind.encode())
    h.update(repr(parts).encode())
    for a in arrays:
        if a is None:
            h.update(b"-")
            continue
        a = np.ascontiguousarray(a)
        h.update(str(a.dtype).encode() + repr(a.shape).encode())
        h.update(a.tobytes())
    return h.hexdigest()


class PrepackCache:
    """Directory of packed-weight blobs (b2m_weight_export), one file per
    (packing kind, attributes, initializer contents)."""

    def __init__(self, ctx, directory: str):
        self.ctx, self.dir = ctx, directory
        os.makedirs(directory, exist_ok=True)
        self.hits = self.misses = 0

    def get_or_make(self, key: str, make, kind: str):
        from .runtime import PackedWeight

        path = os.path.join(self.dir, key + ".b2mw")
        if os.path.exists(path):
            with open(path, "rb") as f:
                blob = f.read()
            h = ctypes.c_void_p()
            buf = ctypes.create_string_buffer(blob, len(blob))
            st = self.ctx.lib.b2m_weight_import(self.ctx.handle, buf, len(blob), ctypes.byref(h))
            if st == 0:
                self.hits += 1
                return PackedWeight(self.ctx, h, kind)
            # A blob of another library version or a damaged file: repack.
        self.misses += 1
        w = make()
        need = ctypes.c_size_t()
        N.check(self.ctx.lib.b2m_weight_export(w.handle, None, 0, ctypes.byref(need)))
        buf = ctypes.create_string_buffer(need.value)
        N.check(self.ctx.lib.b2m_weight_export(w.handle, buf, need.value, ctypes.byref(need)))
        tmp = f"{path}.{os.getpid()}.tmp"
        with open(tmp, "wb") as f:
            f.write(buf.raw)
        os.replace(tmp, path)
        return w


def prepack_session(ctx, model: OnnxModel, cache_dir: str | None = None, f32_mode: int = N.MODE_EXACT,
                    nbits_mode: int = N.MODE_FAST):
    """A dispatch.GpuDispatch for `model` with every MatMul-family initializer
    weight packed now (MatMul / Gemm fp32 B, Gemm transB applied at pack time,
    MatMulInteger / QLinearMatMul int8 B, MatMulNBits b_q + scales + zero
    points, Conv / ConvInteger / QLinearConv weights; ConvTranspose weights
    are uploaded as they are), under the keys the dispatch uses. Returns
    (dispatch, stats)."""
    from . import ops
    from .dispatch import GpuDispatch

    disp = GpuDispatch(ctx, model.initializers, model.elem_types, f32_mode=f32_mode, nbits_mode=nbits_mode)
    cache = PrepackCache(ctx, cache_dir) if cache_dir else None
    inits = model.initializers

    def packed(key, kind, parts, arrays, make):
        if key in disp._packed:
            return
        if cache is None:
            disp._packed[key] = make()
        else:
            pk = "f32" if kind in ("f32", "gemm") else kind
            if kind == "conv":
                pk = "f32" if arrays[0].dtype == np.float32 else "i8"
            w = cache.get_or_make(_cache_key(kind, parts, arrays), make, pk)
            if kind == "conv":  # an imported blob does not carry the ONNX weight shape
                w.shape = tuple(int(d) for d in arrays[0].shape)
            disp._packed[key] = w

    nbits_order = []
    for nd in model.nodes:
        ins = nd.inputs
        if nd.op_type == "MatMul" and len(ins) > 1 and ins[1] in inits and inits[ins[1]].ndim == 2 \
                and inits[ins[1]].dtype == np.float32:
            b = inits[ins[1]]
            packed(("f32", ins[1]), "f32", (), [b], lambda b=b: ctx.prepack_f32(b))
        elif nd.op_type == "Gemm" and len(ins) > 1 and ins[1] in inits and inits[ins[1]].dtype == np.float32:
            b, tb = inits[ins[1]], int(nd.attrs.get("transB", 0)) != 0
            packed(("gemm", ins[1], tb), "gemm", (tb,), [b], lambda b=b, tb=tb: ctx.prepack_f32(b, trans=tb))
        elif nd.op_type in ("MatMulInteger", "QLinearMatMul"):
            bi = 1 if nd.op_type == "MatMulInteger" else 3
            if len(ins) > bi and ins[bi] in inits and inits[ins[bi]].ndim == 2 \
                    and inits[ins[bi]].dtype in (np.int8, np.uint8):
                b = inits[ins[bi]]
                packed(("i8", ins[bi]), "i8", (), [b], lambda b=b: ctx.prepack_i8(b))
        elif nd.op_type in ("Conv", "ConvInteger", "QLinearConv"):
            wi = 3 if nd.op_type == "QLinearConv" else 1
            if len(ins) > wi and ins[wi] in inits and inits[ins[wi]].ndim >= 3 \
                    and inits[ins[wi]].dtype in (np.float32, np.int8, np.uint8):
                wt = inits[ins[wi]]
                packed(("conv", ins[wi]), "conv", (), [wt], lambda wt=wt: ctx.prepack_conv(wt))
        elif nd.op_type == "ConvTranspose" and len(ins) > 1 and ins[1] in inits \
                and inits[ins[1]].dtype == np.float32 and ("convT", ins[1]) not in disp._packed:
            # Read as is by the kernels: uploaded once, nothing to pack or cache.
            disp._packed[("convT", ins[1])] = ctx.upload(np.ascontiguousarray(inits[ins[1]]))
        elif nd.op_type == "MatMulNBits" and len(ins) > 2 and ins[1] in inits and ins[2] in inits:
            k, n = int(nd.attrs["K"]), int(nd.attrs["N"])
            bits, block = int(nd.attrs.get("bits", 4)), int(nd.attrs["block_size"])
            zp_name = ins[3] if len(ins) > 3 else ""
            zp = inits.get(zp_name) if zp_name else None
            bq, sc = inits[ins[1]], inits[ins[2]]
            key = ("nbits", ins[1], ins[2], zp_name)
            packed(key, "nbits", (k, n, bits, block), [bq, sc, zp],
                   lambda bq=bq, sc=sc, zp=zp, k=k, n=n, bits=bits, block=block: ops.prepack_nbits(
                       ctx, bq, sc, zp, k=k, n=n, bits=bits, blockSize=block))
            nbits_order.append(key)
    # The MatMulNBits calls in node order, each weight declared as the
    # successor of the one before (b2m_weight_set_next): their kernels
    # prefetch the next projection's weights into L2.
    for a, b in zip(nbits_order, nbits_order[1:]):
        if a != b:
            disp._packed[a].set_next(disp._packed[b])
    stats = {"packed": len(disp._packed), "cache_hits": cache.hits if cache else 0,
             "cache_misses": cache.misses if cache else 0}
    return disp, stats
