"""CPU compositions of the config-4 (BERT-base) and config-5 (int4 decoder)
chains — TEST INFRASTRUCTURE ONLY (tests/ and bench.py's CPU-baseline leg).

Each composition runs the chain op by op from a dict of host weights, with
this package's restatement of the reference ops:

- MatMul / Gemm: ``oracle.gemm`` / ``oracle.matmul`` (the reference kernel's
  operation order, lib/src/gemm_kernel_simd.dart:32-243).
- MatMulNBits: ``oracle.matmul_nbits`` (lib/src/onnx_qlinear_ops.dart:115-228)
  when ``strict``; otherwise the product of the activations with the weights
  dequantized exactly as the reference's weight() does (:177-191), formed in
  float64 and stored float32. The two differ by float32 accumulation order
  only (~1e-7 relative per op), and the float64 form runs on BLAS, which keeps
  a 28-layer, 512-token composition within seconds.
- RMSNorm, GroupQueryAttention, SiLU*Mul, LayerNorm, MultiHeadAttention and
  GELU: ``oracle.glue``, pinned to the reference's fixtures.

The chains follow the reference executor's node order for these exports
(OnnxGraphExecutor._dispatch, lib/src/onnx_graph.dart:1549): per decoder layer
SkipSimplifiedLayerNormalization, q/k/v MatMulNBits, per-head q/k RMSNorm,
GroupQueryAttention with rotary and past KV, o MatMulNBits, residual RMSNorm,
gate/up MatMulNBits, SiLU*Mul, down MatMulNBits; then the final norm, the fp32
lm_head MatMul. Per encoder layer: QKV Gemm, MultiHeadAttention, O Gemm,
residual LayerNorm, FFN-up Gemm, GELU, FFN-down Gemm, residual LayerNorm.
"""
from __future__ import annotations

import math
import os

import numpy as np

from . import gemm, matmul, matmul_nbits, nbits_dequant
from . import glue

THREADS = os.cpu_count() or 1


def nbits_k(cfg, name):
    return {"qkv": cfg.hidden, "o": cfg.heads * cfg.head_dim, "gate_up": cfg.hidden, "down": cfg.inter}[name]


def nbits_n(cfg, name):
    return {"qkv": (cfg.heads + 2 * cfg.kv_heads) * cfg.head_dim, "o": cfg.hidden, "gate_up": 2 * cfg.inter,
            "down": cfg.hidden}[name]


class DequantCache:
    """Exactly dequantized MatMulNBits weights W[n][k] of a host weight dict,
    made on first use."""

    def __init__(self, cfg, host):
        self.cfg, self.host, self.cache = cfg, host, {}

    def __call__(self, li, name):
        key = (li, name)
        if key not in self.cache:
            bq, sc, zp = self.host[key]
            self.cache[key] = nbits_dequant(bq, sc, zp, nbits_k(self.cfg, name), bq.shape[0], self.cfg.block)
        return self.cache[key]


def nbits_product(a, w):
    """float32(A . W^T) with the product formed in float64 (W exact)."""
    return (np.asarray(a, np.float32).astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)


def decoder_forward(cfg, host, cap, ids, past, strict=True, weights=None, nthreads=THREADS):
    """The decoder chain for int64 ids [B][S] on top of `past` (a list of
    (k, v) per layer, or None). Returns (last-token logits [B][V], new past).
    `strict` runs every MatMulNBits and the lm_head through the oracle
    restatement; otherwise through float64 products (`weights` a
    DequantCache)."""
    c = cfg
    b, s = ids.shape
    t = b * s
    res = host["emb"][ids.reshape(-1)]
    cos, sin = glue.rope_cache(cap, c.head_dim // 2, c.theta)
    newp = []
    down = None

    def mm(x, li, name):
        if strict:
            bq, sc, zp = host[(li, name)]
            return matmul_nbits(x, bq, sc, zp, x.shape[-1], bq.shape[0], c.block, nthreads=nthreads).reshape(t, -1)
        return nbits_product(x, weights(li, name))

    hd = c.head_dim
    for li in range(c.layers):
        if li == 0:
            h, res = glue.rmsnorm(res, host[(li, "attn_norm")], c.eps)
        else:
            h, res = glue.rmsnorm(down, host[(li, "attn_norm")], c.eps, skip=res)
        qkv = mm(h, li, "qkv")
        q = glue.rmsnorm(qkv[:, : c.heads * hd].reshape(-1, hd), host[(li, "q_norm")], c.eps)[0].reshape(t, -1)
        k = glue.rmsnorm(qkv[:, c.heads * hd:(c.heads + c.kv_heads) * hd].reshape(-1, hd), host[(li, "k_norm")],
                         c.eps)[0].reshape(t, -1)
        v = qkv[:, (c.heads + c.kv_heads) * hd:]
        pk, pv = (None, None) if past is None else past[li]
        attn, nk, nv = glue.gqa(q.reshape(b, s, -1), k.reshape(b, s, -1), v.reshape(b, s, -1), c.heads,
                                c.kv_heads, pk, pv, cos, sin)
        newp.append((nk, nv))
        o = mm(attn.reshape(t, -1), li, "o")
        h, res = glue.rmsnorm(o, host[(li, "mlp_norm")], c.eps, skip=res)
        gu = mm(h, li, "gate_up")
        act = glue.silu_mul(gu[:, : c.inter], gu[:, c.inter:])
        down = mm(act, li, "down")
    hf, res = glue.rmsnorm(down, host["final_norm"], c.eps, skip=res)
    last = hf.reshape(b, s, -1)[:, -1]
    if strict:
        logits = matmul(last, host["lm_head"], nthreads=nthreads)
    else:
        logits = (last.astype(np.float64) @ host["lm_head"].astype(np.float64)).astype(np.float32)
    return logits, newp


def bert_forward(cfg, host, ids, mask01, nthreads=THREADS):
    """The encoder chain with the oracle Gemm; returns the last hidden state
    [B*S][H]."""
    c = cfg
    b, s = ids.shape
    t = b * s
    pt = np.tile(host["pos"][:s] + host["typ"][0][None, :], (b, 1)).astype(np.float32)
    x, _ = glue.layernorm(host["word"][ids.reshape(-1)], host["emb_g"], host["emb_b"], c.eps, skip=pt)
    addm = ((1.0 - mask01.astype(np.float32)) * -10000.0).astype(np.float32)
    H = c.hidden
    for li in range(c.layers):
        wq, bq = host[(li, "qkv")]
        qkv = gemm(x, wq, bq, nthreads=nthreads)
        a = glue.mha(qkv[:, :H].reshape(b, s, H), qkv[:, H:2 * H].reshape(b, s, H), qkv[:, 2 * H:].reshape(b, s, H),
                     c.heads, c.heads, addm).reshape(t, H)
        wo, bo = host[(li, "o")]
        h1, _ = glue.layernorm(gemm(a, wo, bo, nthreads=nthreads), *host[(li, "ln1")], c.eps, skip=x)
        w1, b1 = host[(li, "ff1")]
        f = glue.gelu(gemm(h1, w1, b1, nthreads=nthreads))
        w2, b2 = host[(li, "ff2")]
        x, _ = glue.layernorm(gemm(f, w2, b2, nthreads=nthreads), *host[(li, "ln2")], c.eps, skip=h1)
    return x


def decoder_host(cfg, seed=0):
    """Host weights of the config-5 shape with the decoder driver's
    distributions (int4 nibbles uniform, scales |N(0, 0.02)| + 1e-3, packed
    uint4 zero points; norm gains 1 + N(0, 0.1); embeddings N(0, 1); lm_head
    N(0, 1/hidden)), for CPU timing."""
    rng = np.random.default_rng(seed)
    host = {}
    for li in range(cfg.layers):
        for name in ("qkv", "o", "gate_up", "down"):
            k, n = nbits_k(cfg, name), nbits_n(cfg, name)
            nb = (k + cfg.block - 1) // cfg.block
            host[(li, name)] = (rng.integers(0, 256, (n, nb, cfg.block // 2), dtype=np.uint8),
                                (np.abs(rng.standard_normal((n, nb))) * 0.02 + 1e-3).astype(np.float32),
                                rng.integers(0, 256, (n, (nb + 1) // 2), dtype=np.uint8))
        for name, d in (("attn_norm", cfg.hidden), ("mlp_norm", cfg.hidden), ("q_norm", cfg.head_dim),
                        ("k_norm", cfg.head_dim)):
            host[(li, name)] = (1.0 + 0.1 * rng.standard_normal(d)).astype(np.float32)
    host["final_norm"] = (1.0 + 0.1 * rng.standard_normal(cfg.hidden)).astype(np.float32)
    host["emb"] = rng.standard_normal((cfg.vocab, cfg.hidden), dtype=np.float32)
    host["lm_head"] = rng.standard_normal((cfg.hidden, cfg.vocab), dtype=np.float32) / np.float32(math.sqrt(cfg.hidden))
    return host


def bert_host(cfg, seed=0):
    """Host weights of the config-4 shape with the encoder driver's
    distributions (dense ~N(0, 1/fan_in), biases N(0, 0.02), LayerNorm gains
    1 + N(0, 0.1)), for CPU timing."""
    rng = np.random.default_rng(seed)

    def dense(k, n):
        return (rng.standard_normal((k, n), dtype=np.float32) / np.float32(math.sqrt(k))).astype(np.float32)

    def vec(n, base=0.0, sd=0.02):
        return (base + sd * rng.standard_normal(n)).astype(np.float32)

    host = dict(word=rng.standard_normal((cfg.vocab, cfg.hidden), dtype=np.float32),
                pos=rng.standard_normal((cfg.max_pos, cfg.hidden), dtype=np.float32),
                typ=rng.standard_normal((2, cfg.hidden), dtype=np.float32),
                emb_g=vec(cfg.hidden, 1.0, 0.1), emb_b=vec(cfg.hidden, 0.0, 0.1))
    H, I = cfg.hidden, cfg.inter
    for li in range(cfg.layers):
        for name, k, n in (("qkv", H, 3 * H), ("o", H, H), ("ff1", H, I), ("ff2", I, H)):
            host[(li, name)] = (dense(k, n), vec(n))
        for name in ("ln1", "ln2"):
            host[(li, name)] = (vec(H, 1.0, 0.1), vec(H, 0.0, 0.1))
    return host
