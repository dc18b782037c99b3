"""numpy compositions of the config-4 (BERT-base) and config-5 (int4
decoder) chains — TEST INFRASTRUCTURE ONLY.

Each composition runs the chain op by op on the host from the drivers' kept
host weights, with the oracle's restatement of the reference ops:

- MatMul / Gemm: ``oracle.gemm`` (the reference kernel's operation order,
  lib/src/gemm_kernel_simd.dart:32-243).
- MatMulNBits: ``oracle.matmul_nbits`` (lib/src/onnx_qlinear_ops.dart:115-228)
  when ``strict``; otherwise the product of the activations with the weights
  dequantized exactly as the reference's weight() does (:177-191), formed in
  float64 and stored float32. The two differ by float32 accumulation order
  only (~1e-7 relative per op), far below every tolerance they are used with,
  and the float64 form runs on BLAS, which keeps a 28-layer, 512-token
  composition within seconds.
- RMSNorm, GroupQueryAttention, SiLU*Mul, LayerNorm, MultiHeadAttention and
  GELU: ``oracle.glue``, pinned to the reference's fixtures.
"""
from __future__ import annotations

import os

import numpy as np

import oracle
from oracle import glue

THREADS = os.cpu_count() or 1


class NbitsWeights:
    """Exactly dequantized MatMulNBits weights W[n][k] of a decoder's kept
    host weights, made on first use."""

    def __init__(self, dec):
        self.dec = dec
        self.cache = {}

    def __call__(self, li, name):
        key = (li, name)
        if key not in self.cache:
            c = self.dec.cfg
            bq, sc, zp = self.dec.host[key]
            n = bq.shape[0]
            k = {"qkv": c.hidden, "o": c.heads * c.head_dim, "gate_up": c.hidden, "down": c.inter}[name]
            self.cache[key] = oracle.nbits_dequant(bq, sc, zp, k, n, c.block)
        return self.cache[key]


def nbits_product(a, w):
    """float32(A . W^T) with the product formed in float64 (W exact)."""
    return (np.asarray(a, np.float32).astype(np.float64) @ w.astype(np.float64).T).astype(np.float32)


def ref_decoder(dec, ids, past, strict=True, weights=None):
    """The decoder chain for int64 ids [B][S] on top of `past` (a list of
    (k, v) per layer, or None). Returns (last-token logits [B][V], new past).
    `strict` runs every MatMulNBits and the lm_head through the oracle
    restatement; otherwise through float64 products (`weights` an
    NbitsWeights)."""
    c = dec.cfg
    hst = dec.host
    b, s = ids.shape
    t = b * s
    res = hst["emb"][ids.reshape(-1)]
    cos, sin = glue.rope_cache(dec.cap, c.head_dim // 2, c.theta)
    newp = []
    down = None

    def mm(x, li, name):
        if strict:
            bq, sc, zp = hst[(li, name)]
            return oracle.matmul_nbits(x, bq, sc, zp, x.shape[-1], bq.shape[0], c.block,
                                       nthreads=THREADS).reshape(t, -1)
        return nbits_product(x, weights(li, name))

    hd = c.head_dim
    for li in range(c.layers):
        if li == 0:
            h, res = glue.rmsnorm(res, hst[(li, "attn_norm")], c.eps)
        else:
            h, res = glue.rmsnorm(down, hst[(li, "attn_norm")], c.eps, skip=res)
        qkv = mm(h, li, "qkv")
        q = glue.rmsnorm(qkv[:, : c.heads * hd].reshape(-1, hd), hst[(li, "q_norm")], c.eps)[0].reshape(t, -1)
        k = glue.rmsnorm(qkv[:, c.heads * hd:(c.heads + c.kv_heads) * hd].reshape(-1, hd), hst[(li, "k_norm")],
                         c.eps)[0].reshape(t, -1)
        v = qkv[:, (c.heads + c.kv_heads) * hd:]
        pk, pv = (None, None) if past is None else past[li]
        attn, nk, nv = glue.gqa(q.reshape(b, s, -1), k.reshape(b, s, -1), v.reshape(b, s, -1), c.heads,
                                c.kv_heads, pk, pv, cos, sin)
        newp.append((nk, nv))
        o = mm(attn.reshape(t, -1), li, "o")
        h, res = glue.rmsnorm(o, hst[(li, "mlp_norm")], c.eps, skip=res)
        gu = mm(h, li, "gate_up")
        act = glue.silu_mul(gu[:, : c.inter], gu[:, c.inter:])
        down = mm(act, li, "down")
    hf, res = glue.rmsnorm(down, hst["final_norm"], c.eps, skip=res)
    last = hf.reshape(b, s, -1)[:, -1]
    if strict:
        logits = oracle.matmul(last, hst["lm_head"], nthreads=THREADS)
    else:
        logits = (last.astype(np.float64) @ hst["lm_head"].astype(np.float64)).astype(np.float32)
    return logits, newp


def ref_bert(enc, ids, mask01):
    """The encoder chain: the oracle Gemm (the reference fp32 kernel's
    operation order) and the oracle/glue ops. Returns the last hidden state
    [B*S][H]."""
    c, hst = enc.cfg, enc.host
    b, s = ids.shape
    t = b * s
    pt = np.tile(hst["pos"][:s] + hst["typ"][0][None, :], (b, 1)).astype(np.float32)
    x, _ = glue.layernorm(hst["word"][ids.reshape(-1)], hst["emb_g"], hst["emb_b"], c.eps, skip=pt)
    addm = ((1.0 - mask01.astype(np.float32)) * -10000.0).astype(np.float32)
    H = c.hidden
    for li in range(c.layers):
        wq, bq = hst[(li, "qkv")]
        qkv = oracle.gemm(x, wq, bq, nthreads=THREADS)
        a = glue.mha(qkv[:, :H].reshape(b, s, H), qkv[:, H:2 * H].reshape(b, s, H), qkv[:, 2 * H:].reshape(b, s, H),
                     c.heads, c.heads, addm).reshape(t, H)
        wo, bo = hst[(li, "o")]
        h1, _ = glue.layernorm(oracle.gemm(a, wo, bo, nthreads=THREADS), *hst[(li, "ln1")], c.eps, skip=x)
        w1, b1 = hst[(li, "ff1")]
        f = glue.gelu(oracle.gemm(h1, w1, b1, nthreads=THREADS))
        w2, b2 = hst[(li, "ff2")]
        x, _ = glue.layernorm(oracle.gemm(f, w2, b2, nthreads=THREADS), *hst[(li, "ln2")], c.eps, skip=h1)
    return x


def rel_cos(have, want):
    """(max|d| / max|ref|, cosine) in float64."""
    h = np.asarray(have, np.float64).ravel()
    w = np.asarray(want, np.float64).ravel()
    rel = float(np.max(np.abs(h - w)) / max(float(np.max(np.abs(w))), 1e-30))
    cos = float(np.dot(h, w) / np.sqrt(np.dot(h, h) * np.dot(w, w)))
    return rel, cos
