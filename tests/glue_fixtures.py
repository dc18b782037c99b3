"""Runs the reference's glue-op fixtures (tests/golden/, converted from
test/fixtures/ by tests/golden/make_golden.py) through a pluggable set of op
implementations, so the same case logic checks the numpy restatement
(oracle/glue.py) on the CPU and the device ops on the GPU. Each runner
returns {output name: array} for the outputs the fixture records."""
import numpy as np

GLUE_CASES = ["gelu_erf", "skipsimplifiedlayernorm", "standard_rms_axis_-1", "argmax_axis1", "rotary_embedding",
              "gqa_causal", "gqa_kvcache", "gqa_kvcache_rotary", "mha_no_bias", "mha_with_bias"]


def run_case(g, impl):
    """impl: object with gelu, rmsnorm(x, gamma, eps, skip) -> (y, sum),
    argmax_last(x), rotary(x, pos, cos, sin, heads, interleaved),
    gqa(q, k, v, h, kvh, past_k, past_v, cos, sin, scale) -> (out, pk, pv),
    mha(q, k, v, h, bias4d, scale) -> out."""
    op, x, at = g["op_type"], g["arrays"], g["attrs"]
    outs = g["outputs"]
    if op == "Gelu":
        return {outs[0]: impl.gelu(x[0])}
    if op == "SkipSimplifiedLayerNormalization":
        y, s = impl.rmsnorm(x[0], x[2], at.get("epsilon", 1e-5), x[1])
        return {"out0": y, "out3": s}
    if op == "RMSNormalization":
        y, _ = impl.rmsnorm(x[0], np.asarray(x[1]).reshape(-1), at.get("epsilon", 1e-5), None)
        return {outs[0]: y}
    if op == "ArgMax":
        ax = at.get("axis", 0) % x[0].ndim
        moved = np.moveaxis(x[0], ax, -1)
        r = impl.argmax_last(moved)
        return {outs[0]: np.expand_dims(r, ax) if at.get("keepdims", 1) else r}
    if op == "RotaryEmbedding":
        cos, sin = x[2], x[3]
        heads = at.get("num_heads", 0) or x[0].shape[-1] // (2 * cos.shape[-1])
        return {outs[0]: impl.rotary(x[0], x[1], cos, sin, heads, bool(at.get("interleaved", 0)))}
    if op == "GroupQueryAttention":
        h, kvh = at["num_heads"], at["kv_num_heads"]
        cos = x[7] if len(x) > 7 and at.get("do_rotary", 0) else None
        sin = x[8] if cos is not None else None
        out, pk, pv = impl.gqa(x[0], x[1], x[2], h, kvh, x[3], x[4], cos, sin, at.get("scale", 0.0))
        r = {"out0": out}
        if "out1" in g["expected"]:
            r["out1"], r["out2"] = pk, pv
        return r
    if op == "MultiHeadAttention":
        bias = x[5] if len(x) > 5 else None
        return {outs[0]: impl.mha(x[0], x[1], x[2], at["num_heads"], bias, at.get("scale", 0.0))}
    raise KeyError(op)
