"""Qwen3-shaped int4 decoder on the device-resident MatMul path (BASELINE
config 5), driven through the C ABI.

This is the chain the reference runs node by node in
``OnnxGraphExecutor._dispatch`` (lib/src/onnx_graph.dart:1549) for a decoder
export: per layer SkipSimplifiedLayerNormalization, the q/k/v MatMulNBits,
per-head q/k RMSNorm, GroupQueryAttention with rotary and present/past KV
(lib/src/onnx_ops.dart:1844), the o MatMulNBits, the residual, RMSNorm, the
gate/up MatMulNBits, SiLU*Mul, the down MatMulNBits; then the final norm, the
fp32 lm_head MatMul and ArgMax for greedy decoding. Every tensor stays on the
device between ops; the MatMuls are this package's kernels.

Two graph-level choices mirror the reference's own fusion passes: q/k/v are one
MatMulNBits over the concatenated weight columns, and gate/up likewise (the
outputs are column slices of one product, which is what the separate products
are). The KV cache is preallocated to its capacity and written in place (the
reference concatenates past and present per step); the attention reads the
cached length from device memory, so one decode step is captured once as a
CUDA graph and replayed per token, with the argmax of one step feeding the
embedding gather of the next on the device.

Weights are random with config 3's distributions (int4 nibbles uniform,
scales |N(0, 0.02)| + 1e-3, packed uint4 zero points); there is no
checkpoint.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np

from . import _native as N
from .runtime import torch_stream_scope


@dataclass
class DecoderConfig:
    hidden: int = 1024
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    inter: int = 3072
    layers: int = 28
    vocab: int = 151936
    eps: float = 1e-6
    theta: float = 1e6
    block: int = 32

    @classmethod
    def qwen3_0_6b(cls) -> "DecoderConfig":
        return cls()

    @classmethod
    def tiny(cls) -> "DecoderConfig":
        return cls(hidden=128, heads=4, kv_heads=2, head_dim=32, inter=256, layers=2, vocab=1000)

    @property
    def qkv_n(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim


def random_nbits(rng, k: int, n: int, block: int):
    """MatMulNBits operands with config 3's distributions: packed nibbles
    uint8[n, nb, block/2], scales f32[n, nb], packed uint4 zero points
    uint8[n, ceil(nb/2)]."""
    nb = (k + block - 1) // block
    bq = rng.integers(0, 256, (n, nb, block // 2), dtype=np.uint8)
    scales = (np.abs(rng.standard_normal((n, nb))) * 0.02 + 1e-3).astype(np.float32)
    zp = rng.integers(0, 256, (n, (nb + 1) // 2), dtype=np.uint8)
    return bq, scales, zp


def swiglu_row_order(inter: int) -> np.ndarray:
    """Row order of a stacked [gate; up] weight (2 * inter rows) in the
    tile-interleaved layout b2m_matmul_nbits_swiglu_dev takes: per 128-row
    tile t, gate rows 64t .. 64t+63, then up rows 64t .. 64t+63."""
    t = np.arange(inter // 64)[:, None] * 64 + np.arange(64)[None, :]
    return np.concatenate([t, t + inter], axis=1).reshape(-1)


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


class Int4Decoder:
    """Random-weight decoder of shape `cfg` for `batch` sequences with a KV
    cache of `cap` positions; prompts up to `max_prefill` tokens."""

    def __init__(self, ctx, cfg: DecoderConfig, batch: int, cap: int, max_prefill: int, seed: int = 0,
                 keep_host: bool = False, mode: int = N.MODE_FAST, fused: bool = True, session=None,
                 producer_f16: bool = True, fold_qk_norm: bool = True, swiglu_epilogue: bool = True):
        import torch

        if mode not in (N.MODE_FAST, N.MODE_PRECISE, N.MODE_EXACT):
            raise N.ArgumentError("decoder: mode must be FAST, PRECISE or EXACT")
        # MatMulNBits numerics of every projection; the lm_head MatMul runs
        # EXACT in EXACT mode and FAST (bf16-split products) otherwise, and the
        # attention runs the fp32 CUDA-core kernels in EXACT mode.
        self.mode = mode
        # fused: q/k/v as one MatMulNBits over the concatenated weight rows and
        # gate/up likewise (a load-time rewrite of same-input siblings); not
        # fused: the exported graph's seven MatMulNBits per layer, each
        # dispatched on its own with its own output, as
        # OnnxGraphExecutor._dispatch runs them (onnx_graph.dart:2918-2934).
        # The weights are the same either way (the fused weight's rows are the
        # separate weights stacked), so the two compute the same columns.
        self.fused = fused if session is None else False
        # session: an _OnnxSession (from_onnx) whose MatMulNBits nodes are run
        # through GpuDispatch.dispatch; the weights are its prepacked
        # initializers.
        self.session = session
        # producer_f16: where a fused projection takes the FAST tensor-core
        # route, the RMSNorm / SiLU*Mul that produces its input also writes the
        # f16 operand (the bits the GEMM's own conversion forms), so the
        # projection runs without its conversion launch.
        self.producer_f16 = producer_f16
        # fold_qk_norm (fused chains): the q / k head norms go into the
        # attention call (b2m_gqa_qknorm_dev), which at one token per sequence
        # normalises, rotates and appends inside the decode kernel: two
        # launches fewer per layer and step, the same results.
        self.fold_qk_norm = fold_qk_norm
        # swiglu_epilogue (fused chains with random weights): the gate / up
        # weight is packed with tile-interleaved rows and one call
        # (b2m_matmul_nbits_swiglu_dev) writes silu(gate) * up, on the
        # tensor-core route from the GEMM's epilogue: no gate / up rows in
        # memory and no SiLU*Mul launch, the same results.
        self.swiglu = bool(swiglu_epilogue and self.fused and session is None and cfg.inter % 64 == 0)
        self._routes = {}
        self.torch = torch
        self.ctx, self.cfg, self.B, self.cap = ctx, cfg, batch, cap
        self.lib = ctx.lib
        c = cfg
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        self.host = {} if keep_host else None
        if session is None:
            self._random_weights(ctx, seed, keep_host)
        else:
            self._session_weights(session)
        half = c.head_dim // 2
        inv = 1.0 / (c.theta ** (np.arange(half, dtype=np.float64) * 2.0 / c.head_dim))
        ang = np.arange(cap, dtype=np.float64)[:, None] * inv[None, :]
        self.cos = torch.from_numpy(np.cos(ang).astype(np.float32)).to(dev)
        self.sin = torch.from_numpy(np.sin(ang).astype(np.float32)).to(dev)
        kv_shape = (c.layers, batch, c.kv_heads, cap, c.head_dim)
        self.kcache = torch.zeros(kv_shape, device=dev, dtype=torch.float32)
        self.vcache = torch.zeros(kv_shape, device=dev, dtype=torch.float32)
        self.past = torch.zeros(batch, device=dev, dtype=torch.int32)
        t = batch * max_prefill
        self.max_tokens = t
        f32 = dict(device=dev, dtype=torch.float32)
        self.res = torch.empty((t, c.hidden), **f32)
        self.h = torch.empty((t, c.hidden), **f32)
        self.qkv = torch.empty((t, c.qkv_n), **f32)
        if not self.fused:  # separate outputs, one per projection
            self.q = torch.empty((t, c.heads * c.head_dim), **f32)
            self.k = torch.empty((t, c.kv_heads * c.head_dim), **f32)
            self.v = torch.empty((t, c.kv_heads * c.head_dim), **f32)
            self.gate = torch.empty((t, c.inter), **f32)
            self.up = torch.empty((t, c.inter), **f32)
        self.attn = torch.empty((t, c.heads * c.head_dim), **f32)
        self.o = torch.empty((t, c.hidden), **f32)
        if not self.swiglu:
            self.gu = torch.empty((t, 2 * c.inter), **f32)
        self.act = torch.empty((t, c.inter), **f32)
        if self.fused and producer_f16:
            self.h16 = torch.empty((t, c.hidden), device=dev, dtype=torch.float16)
            self.act16 = torch.empty((t, c.inter), device=dev, dtype=torch.float16)
            self.attn16 = torch.empty((t, c.heads * c.head_dim), device=dev, dtype=torch.float16)
        self.down = torch.empty((t, c.hidden), **f32)
        self.last = torch.empty((batch, c.hidden), **f32)
        self.logits = torch.empty((batch, c.vocab), **f32)
        self.ids = torch.zeros(t, device=dev, dtype=torch.int64)
        self.next_ids = torch.zeros(batch, device=dev, dtype=torch.int64)
        self.last_idx = {}
        self.t_last = ctx.wrap(self.last.data_ptr(), (batch, c.hidden), np.float32)
        self.t_logits = ctx.wrap(self.logits.data_ptr(), (batch, c.vocab), np.float32)
        self.graph = None
        self.stream = torch.cuda.Stream(device=dev)
        self._wraps = {}

    def set_mode(self, mode: int) -> None:
        """Switches the numerics mode (FAST, PRECISE or EXACT) of later calls;
        the captured decode graph is dropped and captured again on next use."""
        if mode not in (N.MODE_FAST, N.MODE_PRECISE, N.MODE_EXACT):
            raise N.ArgumentError("decoder: mode must be FAST, PRECISE or EXACT")
        self.mode = mode
        self.graph = None

    # -- the exported graph ----------------------------------------------------
    PROJ = (("q", "hidden", "q_n"), ("k", "hidden", "kv_n"), ("v", "hidden", "kv_n"), ("o", "q_n", "hidden"),
            ("gate", "hidden", "inter"), ("up", "hidden", "inter"), ("down", "inter", "hidden"))

    def export_onnx(self, path: str) -> None:
        """Writes this decoder (built with keep_host=True) as an ONNX graph in
        the node order of a decoder export run by OnnxGraphExecutor: per layer
        (Skip)SimplifiedLayerNormalization, the q / k / v MatMulNBits, the
        per-head q / k norms, GroupQueryAttention with rotary, the o
        MatMulNBits, SkipSimplifiedLayerNormalization, the gate / up
        MatMulNBits, Sigmoid and the two Muls of SwiGLU, the down MatMulNBits;
        then the final norm and the fp32 lm_head MatMul. The projection
        weights are the separate (unfused) initializers."""
        from . import onnx_writer as W

        if self.host is None or "lm_head" not in self.host:
            raise N.ArgumentError("decoder export: build the decoder with keep_host=True")
        c, hst = self.cfg, self.host
        dims = {"hidden": c.hidden, "q_n": c.heads * c.head_dim, "kv_n": c.kv_heads * c.head_dim, "inter": c.inter}
        rows = {"q": (0, dims["q_n"]), "k": (dims["q_n"], dims["q_n"] + dims["kv_n"]),
                "v": (dims["q_n"] + dims["kv_n"], c.qkv_n), "gate": (0, c.inter), "up": (c.inter, 2 * c.inter)}
        src = {"q": "qkv", "k": "qkv", "v": "qkv", "o": "o", "gate": "gate_up", "up": "gate_up", "down": "down"}
        inits, nodes = [], []
        ms = "com.microsoft"
        inits.append(W.tensor("embed_tokens.weight", hst["emb"]))
        nodes.append(W.node("Gather", ["embed_tokens.weight", "input_ids"], ["x0"]))
        res = "x0"
        prev = None
        eps = W.attr_float("epsilon", c.eps)
        for li in range(c.layers):
            for nm in ("attn_norm", "mlp_norm", "q_norm", "k_norm"):
                inits.append(W.tensor(f"layers.{li}.{nm}.weight", hst[(li, nm)]))
            pre = f"l{li}."
            if prev is None:
                nodes.append(W.node("SimplifiedLayerNormalization", [res, f"layers.{li}.attn_norm.weight"],
                                    [pre + "hn"], [eps]))
            else:
                nodes.append(W.node("SkipSimplifiedLayerNormalization", [prev, res, f"layers.{li}.attn_norm.weight"],
                                    [pre + "hn", "", "", pre + "res0"], [eps], domain=ms))
                res = pre + "res0"
            for part, kd, nd in self.PROJ:
                bq, sc, zp = hst[(li, src[part])]
                r0, r1 = rows.get(part, (0, bq.shape[0]))
                base = f"layers.{li}.{part}"
                inits.append(W.tensor(base + ".qweight", np.ascontiguousarray(bq[r0:r1])))
                inits.append(W.tensor(base + ".scales", np.ascontiguousarray(sc[r0:r1])))
                inits.append(W.tensor(base + ".qzeros", np.ascontiguousarray(zp[r0:r1])))
                x_in = {"q": pre + "hn", "k": pre + "hn", "v": pre + "hn", "o": pre + "attn", "gate": pre + "hn2",
                        "up": pre + "hn2", "down": pre + "act"}[part]
                attrs = [W.attr_int("K", dims[kd]), W.attr_int("N", dims[nd]), W.attr_int("bits", 4),
                         W.attr_int("block_size", c.block)]
                nodes.append(W.node("MatMulNBits", [x_in, base + ".qweight", base + ".scales", base + ".qzeros"],
                                    [pre + part], attrs, domain=ms))
                if part == "v":
                    for h, nm in (("q", "q_norm"), ("k", "k_norm")):
                        nodes.append(W.node("SimplifiedLayerNormalization", [pre + h, f"layers.{li}.{nm}.weight"],
                                            [pre + h + "n"], [eps, W.attr_int("axis", -1)]))
                    nodes.append(W.node("GroupQueryAttention",
                                        [pre + "qn", pre + "kn", pre + "v", f"past_key.{li}", f"past_value.{li}",
                                         "seqlens_k", "total_sequence_length", "cos_cache", "sin_cache"],
                                        [pre + "attn", f"present_key.{li}", f"present_value.{li}"],
                                        [W.attr_int("num_heads", c.heads), W.attr_int("kv_num_heads", c.kv_heads),
                                         W.attr_int("do_rotary", 1)], domain=ms))
                if part == "o":
                    nodes.append(W.node("SkipSimplifiedLayerNormalization",
                                        [pre + "o", res, f"layers.{li}.mlp_norm.weight"],
                                        [pre + "hn2", "", "", pre + "res1"], [eps], domain=ms))
                    res = pre + "res1"
                if part == "up":
                    nodes.append(W.node("Sigmoid", [pre + "gate"], [pre + "sig"]))
                    nodes.append(W.node("Mul", [pre + "gate", pre + "sig"], [pre + "silu"]))
                    nodes.append(W.node("Mul", [pre + "silu", pre + "up"], [pre + "act"]))
            prev = pre + "down"
        inits.append(W.tensor("norm.weight", hst["final_norm"]))
        inits.append(W.tensor("lm_head.weight", hst["lm_head"]))
        nodes.append(W.node("SkipSimplifiedLayerNormalization", [prev, res, "norm.weight"], ["hf"], [eps], domain=ms))
        nodes.append(W.node("MatMul", ["hf", "lm_head.weight"], ["logits"]))
        with open(path, "wb") as f:
            f.write(W.model(nodes, inits, ["input_ids"], ["logits"]))

    @classmethod
    def from_onnx(cls, ctx, path: str, cfg: DecoderConfig, batch: int, cap: int, max_prefill: int,
                  mode: int = N.MODE_FAST, cache_dir: str | None = None) -> "Int4Decoder":
        """A decoder over a model written by export_onnx: load_model reads it,
        prepack_session packs every MatMulNBits / MatMul initializer under the
        keys GpuDispatch looks up (and declares the projections' order for the
        L2 prefetch), and every projection of the chain is run by
        GpuDispatch.dispatch on the node's own inputs and attributes, writing
        into the decoder's buffers. The glue between them (norms, attention,
        SwiGLU) runs as the decoder's device ops."""
        from .onnx_model import load_model, prepack_session

        model = load_model(path)
        disp, _ = prepack_session(ctx, model, cache_dir=cache_dir, nbits_mode=mode)
        sess = _OnnxSession(model, disp, cfg)
        return cls(ctx, cfg, batch, cap, max_prefill, mode=mode, session=sess)

    def _dispatch_proj(self, part: str, lw, x, T: int, y):
        """One MatMulNBits node through the dispatch, into buffer y."""
        node = lw["nodes"][part]
        k, n = int(node.attrs["K"]), int(node.attrs["N"])
        key = (x.data_ptr(), y.data_ptr(), T, k, n)
        pair = self._wraps.get(key)
        if pair is None:
            pair = (self.ctx.wrap(x.data_ptr(), (T, k), np.float32), self.ctx.wrap(y.data_ptr(), (T, n), np.float32))
            self._wraps[key] = pair
        inits = self.session.model.initializers
        vals = [pair[0]] + [inits.get(nm) if nm else None for nm in node.inputs[1:]]
        self.session.dispatch.nbits_mode = self.mode
        self.session.dispatch.dispatch("MatMulNBits", node.inputs, vals, node.attrs, outputs=[pair[1]])

    def _random_weights(self, ctx, seed: int, keep_host: bool):
        """Random weights with config 3's distributions, prepacked."""
        import torch

        c, dev, fused = self.cfg, self.dev, self.fused
        rng = np.random.default_rng(seed)
        self.layers = []
        for li in range(c.layers):
            lw = {}
            for name, k, n in (("qkv", c.hidden, c.qkv_n), ("o", c.heads * c.head_dim, c.hidden),
                               ("gate_up", c.hidden, 2 * c.inter), ("down", c.inter, c.hidden)):
                bq, sc, zp = random_nbits(rng, k, n, c.block)
                if name == "gate_up" and self.swiglu:
                    r = swiglu_row_order(c.inter)
                    lw[name] = ctx.prepack_nbits(np.ascontiguousarray(bq[r]), np.ascontiguousarray(sc[r]),
                                                 np.ascontiguousarray(zp[r]), k, n, 4, c.block)
                elif fused or name in ("o", "down"):
                    lw[name] = ctx.prepack_nbits(bq, sc, zp, k, n, 4, c.block)
                else:
                    splits = ({"q": (0, c.heads * c.head_dim),
                               "k": (c.heads * c.head_dim, (c.heads + c.kv_heads) * c.head_dim),
                               "v": ((c.heads + c.kv_heads) * c.head_dim, c.qkv_n)} if name == "qkv"
                              else {"gate": (0, c.inter), "up": (c.inter, 2 * c.inter)})
                    for part, (r0, r1) in splits.items():
                        lw[part] = ctx.prepack_nbits(np.ascontiguousarray(bq[r0:r1]), np.ascontiguousarray(sc[r0:r1]),
                                                     np.ascontiguousarray(zp[r0:r1]), k, r1 - r0, 4, c.block)
                if keep_host:
                    self.host[(li, name)] = (bq, sc, zp)
            for name, d in (("attn_norm", c.hidden), ("mlp_norm", c.hidden), ("q_norm", c.head_dim),
                            ("k_norm", c.head_dim)):
                g = (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32)
                lw[name] = torch.from_numpy(g).to(dev)
                if keep_host:
                    self.host[(li, name)] = g
            lw["qk_gain"] = self._qk_gain(lw)
            self.layers.append(lw)
        # The projections in call order, each declared as the successor of the
        # one before (the last layer's down projection is followed by the
        # first layer's q/k/v projection of the next step).
        order = ("qkv", "o", "gate_up", "down") if fused else ("q", "k", "v", "o", "gate", "up", "down")
        seq = [lw[nm] for lw in self.layers for nm in order]
        for a, b in zip(seq, seq[1:] + seq[:1]):
            a.set_next(b)
        gf = (1.0 + 0.1 * rng.standard_normal(c.hidden)).astype(np.float32)
        self.final_norm = torch.from_numpy(gf).to(dev)
        gen = torch.Generator(device=dev)
        gen.manual_seed(seed)
        self.emb = torch.randn((c.vocab, c.hidden), generator=gen, device=dev, dtype=torch.float32)
        lm = (rng.standard_normal((c.hidden, c.vocab), dtype=np.float32) / np.float32(math.sqrt(c.hidden)))
        self.lm_head = ctx.prepack_f32(lm)
        if keep_host:
            self.host["final_norm"] = gf
            self.host["emb"] = self.emb.cpu().numpy()
            self.host["lm_head"] = lm
        del lm

    def _qk_gain(self, lw):
        """[heads + kv_heads][head_dim] gains: the q norm's for every query head,
        then the k norm's for every kv head (one launch normalises both)."""
        c = self.cfg
        return self.torch.cat([lw["q_norm"].reshape(1, -1).repeat(c.heads, 1),
                               lw["k_norm"].reshape(1, -1).repeat(c.kv_heads, 1)]).contiguous()

    def _session_weights(self, sess):
        """The weights of an exported model: the MatMulNBits initializers
        packed by prepack_session (looked up under the dispatch's keys), the
        norm gains, the embedding and the lm_head as initializers."""
        import torch

        c, dev, inits = self.cfg, self.dev, sess.model.initializers
        t = lambda name: torch.from_numpy(np.ascontiguousarray(inits[name], np.float32)).to(dev)
        self.layers = []
        for li in range(c.layers):
            lw = {name: t(f"layers.{li}.{name}.weight") for name in ("attn_norm", "mlp_norm", "q_norm", "k_norm")}
            lw["nodes"] = sess.layer_nodes[li]
            lw["qk_gain"] = self._qk_gain(lw)
            self.layers.append(lw)
        self.final_norm = t("norm.weight")
        self.emb = t("embed_tokens.weight")
        self.lm_head = sess.dispatch._packed[("f32", "lm_head.weight")]

    # -- one pass over the layers for `seq` new tokens per sequence -----------
    def _forward(self, seq: int):
        """Runs the chain for the B*seq token ids in self.ids (sequence-major)
        at positions past[b] .. past[b]+seq-1, leaves the logits of each
        sequence's last token in self.logits and its argmax in self.next_ids,
        and advances past by seq. Everything is enqueued on the context's
        stream."""
        self.ctx.set_attention_mode(N.MODE_EXACT if self.mode == N.MODE_EXACT else N.MODE_FAST)
        try:
            self._layers(seq, self.B * seq)
        finally:
            self.ctx.set_attention_mode(N.MODE_FAST)

    def _f16_input(self, w, T: int) -> bool:
        """Whether the fused projection `w` at T rows takes its activations as
        f16 from their producer (FAST mode, tensor-core route)."""
        if not (self.fused and self.producer_f16 and self.session is None and self.mode == N.MODE_FAST):
            return False
        key = (w.handle.value, T)
        r = self._routes.get(key)
        if r is None:
            out = ctypes.c_int32(-1)
            N.check(self.lib.b2m_matmul_nbits_route(self.ctx.handle, w.handle, T, N.MODE_FAST, ctypes.byref(out)))
            r = self._routes[key] = out.value == N.ROUTE_TC_F16 and w.kn[0] % 8 == 0
        return r

    def _norm(self, x, skip, gamma, sum_out, T: int, f16: bool):
        c, lib, h = self.cfg, self.lib, self.ctx.handle
        if f16:  # the projection reads only the f16 rows: no fp32 copy
            N.check(lib.b2m_rmsnorm_f16_dev(h, _ptr(x), skip, _ptr(gamma), None, sum_out, _ptr(self.h16), T,
                                            c.hidden, c.eps))
        else:
            N.check(lib.b2m_rmsnorm_dev(h, _ptr(x), skip, _ptr(gamma), _ptr(self.h), sum_out, T, c.hidden, c.eps))

    def o_input(self, rows: int):
        """fp32 view of the first `rows` rows the last call's o projection read
        (the attention output, widened from its f16 copy where only that was
        written)."""
        if getattr(self, "_o_f16", False):
            return self.attn16[:rows].float()
        return self.attn[:rows]

    def down_input(self, rows: int):
        """fp32 view of the first `rows` rows the last call's down projection
        read: its f16 operand widened where it took one, else the fp32 SiLU*Mul
        output."""
        if getattr(self, "_down_f16", False):
            return self.act16[:rows].float()
        return self.act[:rows]

    def _proj(self, w, T: int, f16: bool, x, x16, y):
        h = self.ctx.handle
        if f16:
            N.check(self.lib.b2m_matmul_nbits_f16_dev(h, _ptr(x16), T, w.handle, None, _ptr(y)))
        else:
            N.check(self.lib.b2m_matmul_nbits_dev(h, _ptr(x), T, w.handle, None, self.mode, _ptr(y)))

    def _layers(self, seq: int, T: int):
        c, lib, h = self.cfg, self.lib, self.ctx.handle
        H, D = c.hidden, c.head_dim
        chk = N.check
        chk(lib.b2m_gather_rows_dev(h, _ptr(self.emb), _ptr(self.ids), _ptr(self.res), T, c.vocab, H))
        qkv = self.qkv.data_ptr()
        q_off, k_off, v_off = 0, c.heads * D * 4, (c.heads + c.kv_heads) * D * 4
        for li, lw in enumerate(self.layers):
            qkv16 = self.fused and self._f16_input(lw["qkv"], T)
            o16 = self.fused and self._f16_input(lw["o"], T)
            gu16 = self.fused and self._f16_input(lw["gate_up"], T)
            dn16 = self.fused and self._f16_input(lw["down"], T)
            self._down_f16 = dn16
            # (with the folded head norms the attention writes only the o
            # projection's f16 operand when that is what it reads)
            self._o_f16 = o16 and self.fold_qk_norm
            if li == 0:
                self._norm(self.res, None, lw["attn_norm"], None, T, qkv16)
            else:  # residual of the previous layer's MLP, then the attention norm
                self._norm(self.down, _ptr(self.res), lw["attn_norm"], _ptr(self.res), T, qkv16)
            if self.fused:
                self._proj(lw["qkv"], T, qkv16, self.h, getattr(self, "h16", None), self.qkv)
                qp, kp, vp = qkv + q_off, qkv + k_off, qkv + v_off
                q_rs = kv_rs = c.qkv_n
            else:
                for part in ("q", "k", "v"):
                    if self.session is not None:
                        self._dispatch_proj(part, lw, self.h, T, getattr(self, part))
                    else:
                        chk(lib.b2m_matmul_nbits_dev(h, _ptr(self.h), T, lw[part].handle, None, self.mode,
                                                     _ptr(getattr(self, part))))
                qp, kp, vp = self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr()
                q_rs, kv_rs = c.heads * D, c.kv_heads * D
            if self.fused and self.fold_qk_norm:  # head norms inside the attention call
                chk(lib.b2m_gqa_qknorm_dev(h, ctypes.c_void_p(qp), ctypes.c_void_p(kp), ctypes.c_void_p(vp), q_rs,
                                           kv_rs, _ptr(lw["qk_gain"]), c.eps, _ptr(self.kcache[li]),
                                           _ptr(self.vcache[li]), _ptr(self.past), _ptr(self.cos), _ptr(self.sin),
                                           D // 2, D, 0, None if o16 else _ptr(self.attn),
                                           _ptr(self.attn16) if o16 else None, self.B, seq, c.heads, c.kv_heads, D,
                                           self.cap, 0.0))
            else:
                if self.fused:  # q and k heads are adjacent in the packed rows: one launch
                    chk(lib.b2m_rmsnorm_head_rows_dev(h, ctypes.c_void_p(qp), _ptr(lw["qk_gain"]), ctypes.c_void_p(qp),
                                                      T, c.heads + c.kv_heads, D, q_rs, c.eps))
                else:
                    chk(lib.b2m_rmsnorm_heads_dev(h, ctypes.c_void_p(qp), _ptr(lw["q_norm"]), ctypes.c_void_p(qp), T,
                                                  c.heads, D, q_rs, c.eps))
                    chk(lib.b2m_rmsnorm_heads_dev(h, ctypes.c_void_p(kp), _ptr(lw["k_norm"]), ctypes.c_void_p(kp), T,
                                                  c.kv_heads, D, kv_rs, c.eps))
                if o16:  # the attention also writes the o projection's f16 operand
                    chk(lib.b2m_gqa_f16_dev(h, ctypes.c_void_p(qp), ctypes.c_void_p(kp), ctypes.c_void_p(vp), q_rs,
                                            kv_rs, _ptr(self.kcache[li]), _ptr(self.vcache[li]), _ptr(self.past),
                                            _ptr(self.cos), _ptr(self.sin), D // 2, D, 0, _ptr(self.attn),
                                            _ptr(self.attn16), self.B, seq, c.heads, c.kv_heads, D, self.cap, 0.0))
                else:
                    chk(lib.b2m_gqa_dev(h, ctypes.c_void_p(qp), ctypes.c_void_p(kp), ctypes.c_void_p(vp), q_rs, kv_rs,
                                        _ptr(self.kcache[li]), _ptr(self.vcache[li]), _ptr(self.past), _ptr(self.cos),
                                        _ptr(self.sin), D // 2, D, 0, _ptr(self.attn), self.B, seq, c.heads,
                                        c.kv_heads, D, self.cap, 0.0))
            if self.session is not None:
                self._dispatch_proj("o", lw, self.attn, T, self.o)
            else:
                self._proj(lw["o"], T, o16, self.attn, getattr(self, "attn16", None), self.o)
            self._norm(self.o, _ptr(self.res), lw["mlp_norm"], _ptr(self.res), T, gu16)
            if self.swiglu:  # gate / up and SiLU*Mul in one call (tile-interleaved weight rows)
                chk(lib.b2m_matmul_nbits_swiglu_dev(h, _ptr(self.h), _ptr(self.h16) if gu16 else None, T,
                                                    lw["gate_up"].handle, self.mode, None if dn16 else _ptr(self.act),
                                                    _ptr(self.act16) if dn16 else None))
            else:
                if self.fused:
                    self._proj(lw["gate_up"], T, gu16, self.h, getattr(self, "h16", None), self.gu)
                    gp, up_, g_rs = self.gu.data_ptr(), self.gu.data_ptr() + c.inter * 4, 2 * c.inter
                else:
                    for part in ("gate", "up"):
                        if self.session is not None:
                            self._dispatch_proj(part, lw, self.h, T, getattr(self, part))
                        else:
                            chk(lib.b2m_matmul_nbits_dev(h, _ptr(self.h), T, lw[part].handle, None, self.mode,
                                                         _ptr(getattr(self, part))))
                    gp, up_, g_rs = self.gate.data_ptr(), self.up.data_ptr(), c.inter
                # the export's Sigmoid / Mul / Mul nodes as one op, then its down MatMulNBits
                if dn16:
                    chk(lib.b2m_silu_mul_f16_dev(h, ctypes.c_void_p(gp), ctypes.c_void_p(up_), g_rs, g_rs,
                                                 _ptr(self.act), _ptr(self.act16), T, c.inter))
                else:
                    chk(lib.b2m_silu_mul_dev(h, ctypes.c_void_p(gp), ctypes.c_void_p(up_), g_rs, g_rs, _ptr(self.act),
                                             T, c.inter))
            if self.session is not None:
                self._dispatch_proj("down", lw, self.act, T, self.down)
            else:
                self._proj(lw["down"], T, dn16, self.act, getattr(self, "act16", None), self.down)
        chk(lib.b2m_rmsnorm_dev(h, _ptr(self.down), _ptr(self.res), _ptr(self.final_norm), _ptr(self.h),
                                _ptr(self.res), T, H, c.eps))
        idx = self.last_idx.get(seq)
        if idx is None:
            idx = self.torch.arange(self.B, device=self.dev, dtype=self.torch.int64) * seq + (seq - 1)
            self.last_idx[seq] = idx
        chk(lib.b2m_gather_rows_dev(h, _ptr(self.h), _ptr(idx), _ptr(self.last), self.B, T, H))
        y = ctypes.c_void_p(self.t_logits.handle.value)
        lm_mode = N.MODE_EXACT if self.mode == N.MODE_EXACT else N.MODE_FAST
        chk(lib.b2m_matmul_f32(h, self.t_last.handle, None, self.lm_head.handle, lm_mode, ctypes.byref(y)))
        chk(lib.b2m_argmax_dev(h, _ptr(self.logits), _ptr(self.next_ids), self.B, c.vocab))
        chk(lib.b2m_advance_positions_dev(h, _ptr(self.past), self.B, seq))

    def prefill(self, prompt_ids) -> None:
        """prompt_ids: int64 [B][S] (host or device). Resets the cache positions,
        runs the prompt and leaves the first generated token in next_ids."""
        torch = self.torch
        ids = torch.as_tensor(prompt_ids, dtype=torch.int64).to(self.dev).reshape(-1)
        seq = ids.numel() // self.B
        if ids.numel() != self.B * seq or ids.numel() > self.max_tokens or seq > self.cap:
            raise N.ArgumentError("decoder prefill: prompt shape does not fit the decoder")
        with torch_stream_scope(self.ctx, torch, self.stream):
            self.past.zero_()
            self.ids[: ids.numel()].copy_(ids)
            self._forward(seq)

    def _decode_body(self):
        self.ids[: self.B].copy_(self.next_ids)
        self._forward(1)

    def decode(self, steps: int, use_graph: bool = True):
        """Greedy decode `steps` tokens (device-resident loop); returns the
        generated ids as an int64 tensor [steps][B] on the device."""
        torch = self.torch
        with torch_stream_scope(self.ctx, torch, self.stream) as stream:
            out = torch.empty((steps, self.B), device=self.dev, dtype=torch.int64)
            if use_graph and self.graph is None:
                # Capture one step; a warm-up step first so every kernel
                # attribute and scratch size is settled outside the capture.
                # The warm-up's cache writes and position advance are undone.
                saved = self.past.clone()
                self._decode_body()
                self.past.copy_(saved)
                self.next_ids.copy_(self.ids[: self.B])
                g = torch.cuda.CUDAGraph()
                cap_stream = torch.cuda.Stream(device=self.dev)
                cap_stream.wait_stream(stream)
                with torch.cuda.stream(cap_stream):
                    with torch.cuda.graph(g, stream=cap_stream):
                        self.ctx.set_stream(torch.cuda.current_stream().cuda_stream)
                        self._decode_body()
                stream.wait_stream(cap_stream)
                self.ctx.set_stream(stream.cuda_stream)
                self.graph = g
            for i in range(steps):
                if use_graph:
                    self.graph.replay()
                else:
                    self._decode_body()
                out[i].copy_(self.next_ids)
        return out


class _OnnxSession:
    """An exported decoder model, its GpuDispatch, and each layer's
    MatMulNBits nodes by projection name (read from the initializer names
    export_onnx writes: layers.<i>.<proj>.qweight)."""

    def __init__(self, model, dispatch, cfg: DecoderConfig):
        self.model, self.dispatch = model, dispatch
        self.layer_nodes = [dict() for _ in range(cfg.layers)]
        for nd in model.nodes:
            if nd.op_type != "MatMulNBits" or len(nd.inputs) < 2:
                continue
            parts = nd.inputs[1].split(".")
            if len(parts) == 4 and parts[0] == "layers" and parts[3] == "qweight":
                self.layer_nodes[int(parts[1])][parts[2]] = nd
        for li, nodes in enumerate(self.layer_nodes):
            missing = {p for p, _, _ in Int4Decoder.PROJ} - set(nodes)
            if missing:
                raise N.ArgumentError(f"decoder model: layer {li} lacks MatMulNBits nodes {sorted(missing)}")

