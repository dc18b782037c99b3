"""A minimal ONNX protobuf writer: ModelProto bytes with the field numbers of
the ONNX schema (onnx_model.py reads them back). Used to export the drivers'
random-weight models as ONNX graphs and by the loader tests; no onnx package
is needed."""
import struct

import numpy as np


def _varint(v):
    v &= (1 << 64) - 1
    out = bytearray()
    while True:
        b = v & 0x7F
        v >>= 7
        if v:
            out.append(b | 0x80)
        else:
            out.append(b)
            return bytes(out)


def _key(fn, wt):
    return _varint((fn << 3) | wt)


def f_varint(fn, v):
    return _key(fn, 0) + _varint(v)


def f_bytes(fn, b):
    if isinstance(b, str):
        b = b.encode()
    return _key(fn, 2) + _varint(len(b)) + b


def f_float(fn, v):
    return _key(fn, 5) + struct.pack("<f", v)


DT = {np.dtype(np.float32): 1, np.dtype(np.uint8): 2, np.dtype(np.int8): 3, np.dtype(np.int32): 6,
      np.dtype(np.int64): 7, np.dtype(np.float16): 10, np.dtype(np.float64): 11}


def tensor(name, arr, mode="raw", data_type=None, external=None):
    """TensorProto bytes. mode: 'raw' (raw_data), 'typed' (float_data /
    int32_data / int64_data), 'external' (external = (location, offset,
    length))."""
    arr = np.asarray(arr)
    dt = data_type or DT[arr.dtype]
    out = b"".join(f_varint(1, d) for d in arr.shape) + f_varint(2, dt) + f_bytes(8, name)
    if mode == "raw":
        out += f_bytes(9, arr.tobytes())
    elif mode == "typed":
        if dt == 1:
            out += f_bytes(4, arr.astype("<f4").tobytes())
        elif dt == 7:
            out += f_bytes(7, b"".join(_varint(int(x)) for x in arr.ravel()))
        else:
            out += f_bytes(5, b"".join(_varint(int(x)) for x in arr.ravel()))
    elif mode == "external":
        loc, off, ln = external
        for k, v in (("location", loc), ("offset", str(off)), ("length", str(ln))):
            out += f_bytes(13, f_bytes(1, k) + f_bytes(2, v))
        out += f_varint(14, 1)
    elif mode == "raw_bytes":
        out += f_bytes(9, bytes(arr))
    return out


def attr_int(name, v):
    return f_bytes(1, name) + f_varint(3, v) + f_varint(20, 2)


def attr_ints(name, values):
    return f_bytes(1, name) + f_bytes(8, b"".join(_varint(int(v)) for v in values)) + f_varint(20, 7)


def attr_float(name, v):
    return f_bytes(1, name) + f_float(2, v) + f_varint(20, 1)


def node(op, inputs, outputs, attrs=(), domain=""):
    out = b"".join(f_bytes(1, i) for i in inputs) + b"".join(f_bytes(2, o) for o in outputs) + f_bytes(4, op)
    out += b"".join(f_bytes(5, a) for a in attrs)
    if domain:
        out += f_bytes(7, domain)
    return out


def value_info(name):
    return f_bytes(1, name)


def model(nodes, initializers, inputs, outputs):
    graph = b"".join(f_bytes(1, n) for n in nodes) + b"".join(f_bytes(5, t) for t in initializers)
    graph += b"".join(f_bytes(11, value_info(i)) for i in inputs) + b"".join(f_bytes(12, value_info(o)) for o in outputs)
    return f_varint(1, 8) + f_bytes(7, graph)
