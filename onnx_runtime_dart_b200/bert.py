"""BERT-shaped fp32 encoder chain, device-resident end to end.

The MatMul chain of an exported BERT encoder as the reference runtime executes
it (opGemm / opMatMul with prepacked initializers, lib/src/onnx_ops.dart:1710,
2152; the fused SDPA between the two attention MatMuls, :2106-2148;
opLayerNormalization :1666; erf GELU :706), with every intermediate kept in
device memory:

    x   = LayerNorm(word[ids] + position[s] + token_type[0])
    per layer:
      qkv = x . Wqkv + bqkv                    (the Q, K and V Gemms as one)
      a   = softmax(q k^T / sqrt(d) + mask) v  (b2m_mha_dev)
      h   = LayerNorm(a . Wo + bo + x)
      x   = LayerNorm(gelu(h . W1 + b1) . W2 + b2 + h)

Q, K and V share one packed [hidden, 3*hidden] weight: every output column of
a MatMul is computed independently, so concatenating the three weights along
N gives the same three outputs and fills three times more SMs per launch.
Weights are random (seeded, ~N(0, 1/fan_in)); there is no model file.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import numpy as np

from . import _native as N
from .runtime import torch_stream_scope


@dataclass
class BertConfig:
    layers: int = 12
    hidden: int = 768
    heads: int = 12
    inter: int = 3072
    vocab: int = 30522
    max_pos: int = 512
    eps: float = 1e-12

    @classmethod
    def base(cls) -> "BertConfig":
        return cls()

    @classmethod
    def tiny(cls) -> "BertConfig":
        return cls(layers=2, hidden=128, heads=4, inter=512, vocab=1000, max_pos=64)

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    def flops_per_token(self, seq: int) -> int:
        """Linear FLOPs (QKV, O, FFN) plus the two attention MatMuls, per token."""
        lin = 2 * (4 * self.hidden * self.hidden + 2 * self.hidden * self.inter)
        att = 2 * 2 * seq * self.hidden
        return self.layers * (lin + att)


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


class BertEncoder:
    """Random-weight encoder of shape `cfg` for batches of `batch` sequences of
    `seq` tokens. `mode` is the MatMul mode (N.MODE_FAST: bf16-split products on the tensor cores;
    N.MODE_EXACT: the reference's fp32 operation order, with the attention on
    the fp32 CUDA-core kernels)."""

    def __init__(self, ctx, cfg: BertConfig, batch: int, seq: int, seed: int = 0, mode: int = N.MODE_FAST,
                 keep_host: bool = False, producer_split: bool = True):
        import torch

        if seq > cfg.max_pos:
            raise N.ArgumentError("BertEncoder: seq exceeds max_pos")
        self.torch = torch
        self.ctx, self.cfg, self.B, self.S, self.mode = ctx, cfg, batch, seq, mode
        # producer_split (FAST mode): the LayerNorms and the GELU in front of
        # the QKV, FFN-up and FFN-down Gemms also write the bf16 hi / lo planes
        # those Gemms take (the bits of the GEMM's own split), so each runs
        # without its split pass; the GELU then writes only the planes.
        self.split = producer_split and mode == N.MODE_FAST and cfg.hidden % 64 == 0 and cfg.inter % 64 == 0
        self.lib = ctx.lib
        c = cfg
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        rng = np.random.default_rng(seed)
        self.host = {} if keep_host else None
        f32 = dict(device=dev, dtype=torch.float32)
        T = batch * seq
        self.T = T

        def dense(k, n):
            return (rng.standard_normal((k, n), dtype=np.float32) / np.float32(math.sqrt(k))).astype(np.float32)

        def vec(n, base=0.0, sd=0.02):
            return (base + sd * rng.standard_normal(n)).astype(np.float32)

        word = rng.standard_normal((c.vocab, c.hidden), dtype=np.float32)
        pos = rng.standard_normal((c.max_pos, c.hidden), dtype=np.float32)
        typ = rng.standard_normal((2, c.hidden), dtype=np.float32)
        eg, eb = vec(c.hidden, 1.0, 0.1), vec(c.hidden, 0.0, 0.1)
        self.word = torch.from_numpy(word).to(dev)
        # position[s] + token_type[0] for every token of a batch, as one skip
        # operand of the embedding LayerNorm.
        pt = (pos[:seq] + typ[0][None, :]).astype(np.float32)
        self.pos_type = torch.from_numpy(np.tile(pt, (batch, 1))).to(dev)
        self.emb_g, self.emb_b = torch.from_numpy(eg).to(dev), torch.from_numpy(eb).to(dev)
        if keep_host:
            self.host.update(word=word, pos=pos, typ=typ, emb_g=eg, emb_b=eb)
        self.layers = []
        H, I = c.hidden, c.inter
        for li in range(c.layers):
            lw = {}
            for name, k, n in (("qkv", H, 3 * H), ("o", H, H), ("ff1", H, I), ("ff2", I, H)):
                w, b = dense(k, n), vec(n)
                lw[name] = ctx.prepack_f32(w)
                lw[name + "_b"] = torch.from_numpy(b).to(dev)
                if keep_host:
                    self.host[(li, name)] = (w, b)
            for name in ("ln1", "ln2"):
                g, bb = vec(H, 1.0, 0.1), vec(H, 0.0, 0.1)
                lw[name + "_g"], lw[name + "_b"] = torch.from_numpy(g).to(dev), torch.from_numpy(bb).to(dev)
                if keep_host:
                    self.host[(li, name)] = (g, bb)
            lw["t_qkv_b"] = ctx.wrap(lw["qkv_b"].data_ptr(), (3 * H,), np.float32)
            lw["t_o_b"] = ctx.wrap(lw["o_b"].data_ptr(), (H,), np.float32)
            lw["t_ff1_b"] = ctx.wrap(lw["ff1_b"].data_ptr(), (I,), np.float32)
            lw["t_ff2_b"] = ctx.wrap(lw["ff2_b"].data_ptr(), (H,), np.float32)
            self.layers.append(lw)
        self.x = torch.empty((T, H), **f32)
        self.qkv = torch.empty((T, 3 * H), **f32)
        self.attn = torch.empty((T, H), **f32)
        self.o = torch.empty((T, H), **f32)
        self.h1 = torch.empty((T, H), **f32)
        self.f = torch.empty((T, I), **f32)
        self.ids = torch.zeros(T, device=dev, dtype=torch.int64)
        self.mask = torch.zeros((batch, seq), **f32)
        if self.split:  # [2][rows][d] bf16: hi plane, then lo plane
            self.xs = torch.empty((2, T, H), device=dev, dtype=torch.bfloat16)
            self.h1s = torch.empty((2, T, H), device=dev, dtype=torch.bfloat16)
            self.fs = torch.empty((2, T, I), device=dev, dtype=torch.bfloat16)
            self.attns = torch.empty((2, T, H), device=dev, dtype=torch.bfloat16)
        w = ctx.wrap
        self.t = dict(x=w(self.x.data_ptr(), (T, H), np.float32), qkv=w(self.qkv.data_ptr(), (T, 3 * H), np.float32),
                      attn=w(self.attn.data_ptr(), (T, H), np.float32), o=w(self.o.data_ptr(), (T, H), np.float32),
                      h1=w(self.h1.data_ptr(), (T, H), np.float32), f=w(self.f.data_ptr(), (T, I), np.float32))
        self.graph = None
        self.stream = torch.cuda.Stream(device=dev)

    def set_attention_mask(self, attention_mask) -> None:
        """attention_mask [batch][seq] of 0/1 -> additive (1 - m) * -10000, the
        bias a BERT export builds before its attention MatMuls."""
        m = np.asarray(attention_mask, np.float32).reshape(self.B, self.S)
        self.mask.copy_(self.torch.from_numpy(((1.0 - m) * -10000.0).astype(np.float32)))

    def _gemm(self, a, lw, name, y):
        yh = ctypes.c_void_p(self.t[y].handle.value)
        N.check(self.lib.b2m_gemm_f32(self.ctx.handle, self.t[a].handle, None, lw[name].handle,
                                      lw["t_" + name + "_b"].handle, ctypes.c_float(1.0), ctypes.c_float(1.0), 0, 0,
                                      self.mode, ctypes.byref(yh)))

    def _forward(self):
        # EXACT mode also runs the attention on the fp32 CUDA-core kernels.
        self.ctx.set_attention_mode(N.MODE_EXACT if self.mode == N.MODE_EXACT else N.MODE_FAST)
        try:
            self._layers()
        finally:
            self.ctx.set_attention_mode(N.MODE_FAST)

    def _gemm_split(self, planes, lw, name, y):
        N.check(self.lib.b2m_gemm_f32_split_dev(self.ctx.handle, _ptr(planes), self.T, lw[name].handle,
                                                _ptr(lw[name + "_b"]), _ptr(y)))

    def _ln(self, x, skip, g, b, y, planes):
        c, T = self.cfg, self.T
        if planes is not None:
            N.check(self.lib.b2m_layernorm_split_dev(self.ctx.handle, _ptr(x), _ptr(skip), _ptr(g), _ptr(b), _ptr(y),
                                                     None, _ptr(planes), T, c.hidden, ctypes.c_double(c.eps)))
        else:
            N.check(self.lib.b2m_layernorm_dev(self.ctx.handle, _ptr(x), _ptr(skip), _ptr(g), _ptr(b), _ptr(y), None,
                                               T, c.hidden, ctypes.c_double(c.eps)))

    def _layers(self):
        c, lib, h, chk = self.cfg, self.lib, self.ctx.handle, N.check
        T, H, I, D = self.T, c.hidden, c.inter, c.head_dim
        sp = self.split
        chk(lib.b2m_gather_rows_dev(h, _ptr(self.word), _ptr(self.ids), _ptr(self.o), T, c.vocab, H))
        self._ln(self.o, self.pos_type, self.emb_g, self.emb_b, self.x, self.xs if sp else None)
        qkv = self.qkv.data_ptr()
        for lw in self.layers:
            if sp:
                self._gemm_split(self.xs, lw, "qkv", self.qkv)
            else:
                self._gemm("x", lw, "qkv", "qkv")
            q_, k_, v_ = ctypes.c_void_p(qkv), ctypes.c_void_p(qkv + H * 4), ctypes.c_void_p(qkv + 2 * H * 4)
            if sp:  # the attention also writes the O Gemm's planes
                chk(lib.b2m_mha_split_dev(h, q_, k_, v_, 3 * H, 3 * H, _ptr(self.mask), self.S, 0, 0, _ptr(self.attn),
                                          _ptr(self.attns), self.B, self.S, self.S, c.heads, c.heads, D,
                                          ctypes.c_float(0.0), 0))
                self._gemm_split(self.attns, lw, "o", self.o)
            else:
                chk(lib.b2m_mha_dev(h, q_, k_, v_, 3 * H, 3 * H, _ptr(self.mask), self.S, 0, 0, _ptr(self.attn), self.B,
                                    self.S, self.S, c.heads, c.heads, D, ctypes.c_float(0.0), 0))
                self._gemm("attn", lw, "o", "o")
            self._ln(self.o, self.x, lw["ln1_g"], lw["ln1_b"], self.h1, self.h1s if sp else None)
            if sp:
                self._gemm_split(self.h1s, lw, "ff1", self.f)
                chk(lib.b2m_gelu_split_dev(h, _ptr(self.f), None, _ptr(self.fs), T, I))
                self._gemm_split(self.fs, lw, "ff2", self.o)
            else:
                self._gemm("h1", lw, "ff1", "f")
                chk(lib.b2m_gelu_dev(h, _ptr(self.f), _ptr(self.f), T * I))
                self._gemm("f", lw, "ff2", "o")
            self._ln(self.o, self.h1, lw["ln2_g"], lw["ln2_b"], self.x, self.xs if sp else None)

    def forward_device(self, use_graph: bool = True):
        """One forward over the ids already in `self.ids`, ordered on torch's
        current stream; the last hidden state is left in `self.x`
        ([batch*seq, hidden]). With use_graph the chain is captured once as a
        CUDA graph (after an eager warm-up that settles kernel attributes) and
        replayed."""
        torch = self.torch
        with torch_stream_scope(self.ctx, torch, self.stream) as stream:
            if not use_graph:
                self._forward()
                return self.x
            if self.graph is None:
                self._forward()
                g = torch.cuda.CUDAGraph()
                cap_stream = torch.cuda.Stream(device=self.dev)
                cap_stream.wait_stream(stream)
                with torch.cuda.stream(cap_stream):
                    with torch.cuda.graph(g, stream=cap_stream):
                        self.ctx.set_stream(torch.cuda.current_stream().cuda_stream)
                        self._forward()
                stream.wait_stream(cap_stream)
                self.ctx.set_stream(stream.cuda_stream)
                self.graph = g
            self.graph.replay()
        return self.x

    def forward(self, ids, attention_mask=None, out=None, use_graph: bool = True):
        """ids [batch][seq] (host) -> last hidden state [batch*seq, hidden]:
        a numpy array, or copied into `out` (e.g. a pinned host tensor)."""
        torch = self.torch
        if attention_mask is not None:
            self.set_attention_mask(attention_mask)
        src = torch.as_tensor(np.asarray(ids, np.int64).reshape(-1))
        if src.numel() != self.T:
            raise N.ArgumentError("BertEncoder: ids shape does not match batch x seq")
        self.ids.copy_(src, non_blocking=True)
        self.forward_device(use_graph)
        if out is None:
            return self.x.cpu().numpy()
        out.copy_(self.x, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        return out
