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


def _ptr(t) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


class Int4Decoder:
    """Random-weight decoder of shape `cfg` for `batch` sequences with a KV
    cache of `cap` positions; prompts up to `max_prefill` tokens."""

    def __init__(self, ctx, cfg: DecoderConfig, batch: int, cap: int, max_prefill: int, seed: int = 0,
                 keep_host: bool = False, mode: int = N.MODE_FAST, fused: bool = True):
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
        self.fused = fused
        self.torch = torch
        self.ctx, self.cfg, self.B, self.cap = ctx, cfg, batch, cap
        self.lib = ctx.lib
        c = cfg
        dev = torch.device("cuda", torch.cuda.current_device())
        self.dev = dev
        rng = np.random.default_rng(seed)
        self.host = {} if keep_host else None
        self.layers = []
        for li in range(c.layers):
            lw = {}
            for name, k, n in (("qkv", c.hidden, c.qkv_n), ("o", c.heads * c.head_dim, c.hidden),
                               ("gate_up", c.hidden, 2 * c.inter), ("down", c.inter, c.hidden)):
                bq, sc, zp = random_nbits(rng, k, n, c.block)
                if fused or name in ("o", "down"):
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
        if not fused:  # separate outputs, one per projection
            self.q = torch.empty((t, c.heads * c.head_dim), **f32)
            self.k = torch.empty((t, c.kv_heads * c.head_dim), **f32)
            self.v = torch.empty((t, c.kv_heads * c.head_dim), **f32)
            self.gate = torch.empty((t, c.inter), **f32)
            self.up = torch.empty((t, c.inter), **f32)
        self.attn = torch.empty((t, c.heads * c.head_dim), **f32)
        self.o = torch.empty((t, c.hidden), **f32)
        self.gu = torch.empty((t, 2 * c.inter), **f32)
        self.act = torch.empty((t, c.inter), **f32)
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

    def set_mode(self, mode: int) -> None:
        """Switches the numerics mode (FAST, PRECISE or EXACT) of later calls;
        the captured decode graph is dropped and captured again on next use."""
        if mode not in (N.MODE_FAST, N.MODE_PRECISE, N.MODE_EXACT):
            raise N.ArgumentError("decoder: mode must be FAST, PRECISE or EXACT")
        self.mode = mode
        self.graph = None

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

    def _layers(self, seq: int, T: int):
        c, lib, h = self.cfg, self.lib, self.ctx.handle
        H, D = c.hidden, c.head_dim
        chk = N.check
        chk(lib.b2m_gather_rows_dev(h, _ptr(self.emb), _ptr(self.ids), _ptr(self.res), T, c.vocab, H))
        qkv = self.qkv.data_ptr()
        q_off, k_off, v_off = 0, c.heads * D * 4, (c.heads + c.kv_heads) * D * 4
        for li, lw in enumerate(self.layers):
            if li == 0:
                chk(lib.b2m_rmsnorm_dev(h, _ptr(self.res), None, _ptr(lw["attn_norm"]), _ptr(self.h), None, T, H,
                                        c.eps))
            else:  # residual of the previous layer's MLP, then the attention norm
                chk(lib.b2m_rmsnorm_dev(h, _ptr(self.down), _ptr(self.res), _ptr(lw["attn_norm"]), _ptr(self.h),
                                        _ptr(self.res), T, H, c.eps))
            if self.fused:
                chk(lib.b2m_matmul_nbits_dev(h, _ptr(self.h), T, lw["qkv"].handle, None, self.mode, _ptr(self.qkv)))
                qp, kp, vp = qkv + q_off, qkv + k_off, qkv + v_off
                q_rs = kv_rs = c.qkv_n
            else:
                for part in ("q", "k", "v"):
                    chk(lib.b2m_matmul_nbits_dev(h, _ptr(self.h), T, lw[part].handle, None, self.mode,
                                                 _ptr(getattr(self, part))))
                qp, kp, vp = self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr()
                q_rs, kv_rs = c.heads * D, c.kv_heads * D
            chk(lib.b2m_rmsnorm_heads_dev(h, ctypes.c_void_p(qp), _ptr(lw["q_norm"]), ctypes.c_void_p(qp), T,
                                          c.heads, D, q_rs, c.eps))
            chk(lib.b2m_rmsnorm_heads_dev(h, ctypes.c_void_p(kp), _ptr(lw["k_norm"]), ctypes.c_void_p(kp), T,
                                          c.kv_heads, D, kv_rs, c.eps))
            chk(lib.b2m_gqa_dev(h, ctypes.c_void_p(qp), ctypes.c_void_p(kp), ctypes.c_void_p(vp), q_rs, kv_rs,
                                _ptr(self.kcache[li]),
                                _ptr(self.vcache[li]), _ptr(self.past), _ptr(self.cos), _ptr(self.sin), D // 2, D, 0,
                                _ptr(self.attn), self.B, seq, c.heads, c.kv_heads, D, self.cap, 0.0))
            chk(lib.b2m_matmul_nbits_dev(h, _ptr(self.attn), T, lw["o"].handle, None, self.mode, _ptr(self.o)))
            chk(lib.b2m_rmsnorm_dev(h, _ptr(self.o), _ptr(self.res), _ptr(lw["mlp_norm"]), _ptr(self.h),
                                    _ptr(self.res), T, H, c.eps))
            if self.fused:
                chk(lib.b2m_matmul_nbits_dev(h, _ptr(self.h), T, lw["gate_up"].handle, None, self.mode,
                                             _ptr(self.gu)))
                gp, up_, g_rs = self.gu.data_ptr(), self.gu.data_ptr() + c.inter * 4, 2 * c.inter
            else:
                for part in ("gate", "up"):
                    chk(lib.b2m_matmul_nbits_dev(h, _ptr(self.h), T, lw[part].handle, None, self.mode,
                                                 _ptr(getattr(self, part))))
                gp, up_, g_rs = self.gate.data_ptr(), self.up.data_ptr(), c.inter
            chk(lib.b2m_silu_mul_dev(h, ctypes.c_void_p(gp), ctypes.c_void_p(up_), g_rs, g_rs, _ptr(self.act), T,
                                     c.inter))
            chk(lib.b2m_matmul_nbits_dev(h, _ptr(self.act), T, lw["down"].handle, None, self.mode,
                                         _ptr(self.down)))
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
