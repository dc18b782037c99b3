"""Load-time prepack: the ONNX protobuf reader (onnx_runtime_dart_b200/
onnx_model.py) on models written by onnx_runtime_dart_b200/onnx_writer.py. CPU tests check the
tensor decoding rules of the reference's tensorFromProto
(lib/src/onnx_proto_loader.dart:171-299) and external data; the GPU tests
check that load-time packing, with and without the on-disk cache, gives the
same outputs as packing on first use."""
import numpy as np
import pytest

from onnx_runtime_dart_b200 import onnx_model as om
from onnx_runtime_dart_b200 import onnx_writer as W


def _write(tmp_path, name, nodes, inits, inputs, outputs, extra=None):
    if extra:
        for fname, data in extra.items():
            (tmp_path / fname).write_bytes(data)
    p = tmp_path / name
    p.write_bytes(W.model(nodes, inits, inputs, outputs))
    return str(p)


def _nbits_operands(rng, k, n, block):
    nb = (k + block - 1) // block
    bq = rng.integers(0, 256, (n, nb, block // 2), dtype=np.uint8)
    sc = (np.abs(rng.normal(0, 0.02, n * nb)) + 1e-3).astype(np.float32)
    zp = rng.integers(0, 256, n * ((nb + 1) // 2), dtype=np.uint8)
    return bq, sc, zp


def build_model(tmp_path):
    rng = np.random.default_rng(3)
    w1 = rng.standard_normal((16, 24)).astype(np.float32)
    w2 = rng.standard_normal((8, 24)).astype(np.float32)        # Gemm B, transB = 1
    c2 = rng.standard_normal(8).astype(np.float32)
    wq = rng.integers(-127, 128, (16, 12)).astype(np.int8)
    bq, sc, zp = _nbits_operands(rng, 64, 40, 32)
    wc = (rng.standard_normal((4, 3, 3, 3)) * 0.2).astype(np.float32)   # Conv weight
    bc = rng.standard_normal(4).astype(np.float32)
    wi = rng.integers(-127, 128, (5, 2, 3, 3)).astype(np.int8)          # ConvInteger weight
    wt = (rng.standard_normal((3, 2, 2, 2)) * 0.5).astype(np.float32)   # ConvTranspose weight
    pad = b"\0" * 24
    ext = pad + w2.tobytes()
    inits = [W.tensor("w1", w1, "raw"),
             W.tensor("w2", w2, "external", external=("w.bin", len(pad), w2.nbytes)),
             W.tensor("c2", c2, "typed"),
             W.tensor("wq", wq, "typed"),
             W.tensor("bq", bq, "raw"), W.tensor("sc", sc, "raw"), W.tensor("zp", zp, "raw"),
             W.tensor("wc", wc, "raw"), W.tensor("bc", bc, "typed"), W.tensor("wi", wi, "raw"),
             W.tensor("wt", wt, "raw")]
    nodes = [W.node("MatMul", ["x", "w1"], ["y1"]),
             W.node("Gemm", ["x24", "w2", "c2"], ["y2"], [W.attr_int("transB", 1), W.attr_float("alpha", 0.5)]),
             W.node("MatMulInteger", ["xq", "wq"], ["y3"]),
             W.node("MatMulNBits", ["x64", "bq", "sc", "zp"], ["y4"],
                    [W.attr_int("K", 64), W.attr_int("N", 40), W.attr_int("bits", 4), W.attr_int("block_size", 32)],
                    domain="com.microsoft"),
             W.node("Conv", ["xc", "wc", "bc"], ["y5"], [W.attr_ints("pads", [1, 1, 1, 1]),
                                                       W.attr_ints("kernel_shape", [3, 3])]),
             W.node("ConvInteger", ["xi", "wi"], ["y6"], [W.attr_ints("strides", [2, 1])]),
             W.node("ConvTranspose", ["xt", "wt"], ["y7"], [W.attr_ints("strides", [2, 2])])]
    path = _write(tmp_path, "m.onnx", nodes, inits, ["x", "x24", "xq", "x64", "xc", "xi", "xt"],
                  ["y1", "y2", "y3", "y4", "y5", "y6", "y7"], {"w.bin": ext})
    return path, dict(w1=w1, w2=w2, c2=c2, wq=wq, bq=bq, sc=sc, zp=zp, wc=wc, bc=bc, wi=wi, wt=wt)


def test_reads_graph_initializers_and_external_data(tmp_path):
    path, ref = build_model(tmp_path)
    m = om.load_model(path)
    assert [n.op_type for n in m.nodes] == ["MatMul", "Gemm", "MatMulInteger", "MatMulNBits", "Conv", "ConvInteger",
                                            "ConvTranspose"]
    assert m.nodes[1].attrs["transB"] == 1 and abs(m.nodes[1].attrs["alpha"] - 0.5) < 1e-7
    assert m.nodes[3].domain == "com.microsoft" and m.nodes[3].attrs["block_size"] == 32
    assert m.nodes[4].attrs["pads"] == [1, 1, 1, 1] and m.nodes[5].attrs["strides"] == [2, 1]
    for k, v in ref.items():
        np.testing.assert_array_equal(m.initializers[k], v)
        assert m.initializers[k].dtype == v.dtype
    assert m.elem_types["wq"] == om.INT8 and m.elem_types["w2"] == om.FLOAT
    assert m.inputs == ["x", "x24", "xq", "x64", "xc", "xi", "xt"]
    assert m.outputs == ["y1", "y2", "y3", "y4", "y5", "y6", "y7"]


def test_tensor_decoding_rules():
    # float16 widened, double narrowed, int32 / bool carried as int64, int4 /
    # uint4 unpacked low nibble first (sign-extended for int4).
    h = np.array([1.5, -2.25, 65504.0], np.float16)
    t = om.decode_tensor(memoryview(W.tensor("h", h, "raw")))
    assert t.array.dtype == np.float32 and t.array.tolist() == [1.5, -2.25, 65504.0]
    d = np.array([0.1, 2.0], np.float64)
    assert om.decode_tensor(memoryview(W.tensor("d", d, "raw"))).array.dtype == np.float32
    i = np.array([[1, -2], [3, 4]], np.int32)
    t = om.decode_tensor(memoryview(W.tensor("i", i, "raw")))
    assert t.array.dtype == np.int64 and t.array.tolist() == [[1, -2], [3, 4]]
    b = np.array([0, 1, 7], np.uint8)
    t = om.decode_tensor(memoryview(W.tensor("b", b, "raw", data_type=om.BOOL)))
    assert t.array.tolist() == [0, 1, 1]
    packed = bytes([0x21, 0xF8, 0x07])            # 1, 2, 8, 15, 7
    raw4 = W.f_varint(1, 5) + W.f_varint(2, om.INT4) + W.f_bytes(8, "q") + W.f_bytes(9, packed)
    assert om.decode_tensor(memoryview(raw4)).array.tolist() == [1, 2, -8, -1, 7]
    rawu4 = W.f_varint(1, 5) + W.f_varint(2, om.UINT4) + W.f_bytes(8, "q") + W.f_bytes(9, packed)
    assert om.decode_tensor(memoryview(rawu4)).array.tolist() == [1, 2, 8, 15, 7]


def test_malformed_tensors_raise_like_the_reference():
    short = W.f_varint(1, 4) + W.f_varint(2, om.FLOAT) + W.f_bytes(8, "s") + W.f_bytes(9, b"\0" * 8)
    with pytest.raises(ValueError, match="raw_data too short"):
        om.decode_tensor(memoryview(short))
    neg = W.f_varint(1, (1 << 64) - 3) + W.f_varint(2, om.FLOAT) + W.f_bytes(8, "n")
    with pytest.raises(ValueError, match="negative dimension"):
        om.decode_tensor(memoryview(neg))
    inline = W.f_varint(1, 3) + W.f_varint(2, om.FLOAT) + W.f_bytes(8, "i") + W.f_bytes(4, b"\0" * 8)
    with pytest.raises(ValueError, match="inline data length"):
        om.decode_tensor(memoryview(inline))
    ext = W.tensor("e", np.zeros(2, np.float32), "external", external=("x.bin", 0, 8))
    with pytest.raises(RuntimeError, match="externally"):
        om.decode_tensor(memoryview(ext))


@pytest.mark.gpu
def test_load_time_prepack_and_cache_match_first_use_packing(tmp_path):
    torch = pytest.importorskip("torch")  # noqa: F841
    import onnx_runtime_dart_b200 as b2m
    from onnx_runtime_dart_b200 import ops
    from onnx_runtime_dart_b200.dispatch import GpuDispatch

    path, ref = build_model(tmp_path)
    m = om.load_model(path)
    ctx = b2m.Context(0)
    rng = np.random.default_rng(8)
    feeds = {"x": rng.standard_normal((5, 16)).astype(np.float32),
             "x24": rng.standard_normal((6, 24)).astype(np.float32),
             "xq": rng.integers(0, 256, (7, 16), dtype=np.uint8),
             "x64": rng.standard_normal((9, 64)).astype(np.float32),
             "xc": rng.standard_normal((2, 3, 9, 9)).astype(np.float32),
             "xi": rng.integers(0, 256, (1, 2, 7, 7), dtype=np.uint8),
             "xt": rng.standard_normal((1, 3, 4, 5)).astype(np.float32)}

    def run(disp):
        out = []
        for nd in m.nodes:
            vals = [feeds.get(nm, m.initializers.get(nm)) for nm in nd.inputs]
            y = disp.dispatch(nd.op_type, nd.inputs, vals, nd.attrs)[0]
            out.append(y.numpy())
        return out

    lazy = run(GpuDispatch(ctx, m.initializers, m.elem_types))
    eager, st0 = om.prepack_session(ctx, m)
    assert st0["packed"] == 7
    first = run(eager)
    cache = str(tmp_path / "cache")
    d1, st1 = om.prepack_session(ctx, m, cache_dir=cache)
    assert st1["cache_misses"] == 6 and st1["cache_hits"] == 0  # the ConvTranspose weight is uploaded, not cached
    d2, st2 = om.prepack_session(ctx, m, cache_dir=cache)
    assert st2["cache_hits"] == 6 and st2["cache_misses"] == 0
    for a, b_, c, d in zip(lazy, first, run(d1), run(d2)):
        np.testing.assert_array_equal(a, b_)
        np.testing.assert_array_equal(a, c)
        np.testing.assert_array_equal(a, d)
    import oracle
    np.testing.assert_array_equal(lazy[4], oracle.conv_f32(feeds["xc"], ref["wc"], ref["bc"], None, [1, 1, 1, 1]))
    np.testing.assert_array_equal(lazy[5].astype(np.int64), oracle.conv_integer(feeds["xi"], ref["wi"], strides=[2, 1]))
    np.testing.assert_array_equal(lazy[6], oracle.conv_transpose_f32(feeds["xt"], ref["wt"], None, [2, 2]))
    np.testing.assert_array_equal(lazy[2].astype(np.int64),
                                  ops.as_reference_int64(ops.opMatMulInteger(feeds["xq"], ref["wq"], ctx=ctx)))
