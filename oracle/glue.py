"""CPU restatement of the transformer glue ops — TEST INFRASTRUCTURE ONLY.

numpy versions of the reference ops that sit between the MatMuls of the
config-4/5 chains, following the reference's arithmetic (float32 storage,
double where Dart computes in double):

- ``rmsnorm``   opRMSNorm, lib/src/onnx_ops.dart:1771-1800 (+ the residual add
  of SkipSimplifiedLayerNormalization, lib/src/onnx_graph.dart:1793-1800)
- ``layernorm`` opLayerNormalization, lib/src/onnx_ops.dart:1666
- ``rotary``    opRotaryEmbedding, lib/src/onnx_ops.dart:2659-2717
- ``gqa``       opGroupQueryAttention, lib/src/onnx_ops.dart:1844-2012
- ``silu_mul``, ``gelu``, ``argmax`` (opArgMinMax, first maximum wins)

Only tests and the smoke check import this module.
"""
from __future__ import annotations

import math

import numpy as np


def rmsnorm(x, gamma, eps, skip=None):
    """Returns (y, s) with s = x (+ skip) in float32 and
    y = f32(s * (1/sqrt(mean_d(s^2) + eps)) * gamma) computed in double."""
    s = np.asarray(x, np.float32)
    if skip is not None:
        s = (s + np.asarray(skip, np.float32)).astype(np.float32)
    sd = s.astype(np.float64)
    inv = 1.0 / np.sqrt((sd * sd).sum(-1, keepdims=True) / s.shape[-1] + eps)
    return (sd * inv * np.asarray(gamma, np.float64)).astype(np.float32), s


def layernorm(x, gamma, beta, eps, skip=None):
    s = np.asarray(x, np.float32)
    if skip is not None:
        s = (s + np.asarray(skip, np.float32)).astype(np.float32)
    sd = s.astype(np.float64)
    mean = sd.mean(-1, keepdims=True)
    var = ((sd - mean) ** 2).mean(-1, keepdims=True)
    y = (sd - mean) / np.sqrt(var + eps) * np.asarray(gamma, np.float64)
    if beta is not None:
        y = y + np.asarray(beta, np.float64)
    return y.astype(np.float32), s


def silu_mul(gate, up):
    g = np.asarray(gate, np.float64)
    return (g / (1.0 + np.exp(-g)) * np.asarray(up, np.float64)).astype(np.float32)


def gelu(x):
    xd = np.asarray(x, np.float64)
    erf = np.vectorize(math.erf)
    return (0.5 * xd * (1.0 + erf(xd / math.sqrt(2.0)))).astype(np.float32)


def argmax(x):
    """Row argmax over the last axis; numpy's argmax also returns the first
    occurrence of the maximum."""
    return np.argmax(np.asarray(x, np.float32), axis=-1).astype(np.int64)


def rope_cache(max_pos, half, theta):
    """cos / sin caches [max_pos][half] as float32 (inv_freq = theta^(-2i/dim))."""
    inv = 1.0 / (theta ** (np.arange(half, dtype=np.float64) * 2.0 / (2 * half)))
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def rotary(x, positions, cos, sin, num_heads, interleaved=False):
    """x: [B][S][H*D] float32, positions: [B][S] int. Rotated in double, stored
    float32 (opRotaryEmbedding)."""
    x = np.asarray(x, np.float32)
    b, s, hid = x.shape
    d = hid // num_heads
    half = cos.shape[-1]
    rot = 2 * half
    xv = x.reshape(b, s, num_heads, d).astype(np.float64)
    out = xv.copy()
    c = cos[np.asarray(positions)].astype(np.float64)[:, :, None, :]  # [B][S][1][half]
    sn = sin[np.asarray(positions)].astype(np.float64)[:, :, None, :]
    if interleaved:
        x0, x1 = xv[..., 0:rot:2], xv[..., 1:rot:2]
        out[..., 0:rot:2] = x0 * c - x1 * sn
        out[..., 1:rot:2] = x1 * c + x0 * sn
    else:
        x0, x1 = xv[..., :half], xv[..., half:rot]
        out[..., :half] = x0 * c - x1 * sn
        out[..., half:rot] = x1 * c + x0 * sn
    return out.astype(np.float32).reshape(b, s, hid)


def gqa(q, k, v, num_heads, kv_heads, past_k=None, past_v=None, cos=None, sin=None, scale=None,
        interleaved=False):
    """opGroupQueryAttention: q [B][S][H*D], k / v [B][S][KVH*D], past [B][KVH][P][D].
    Returns (out [B][S][H*D], present_k, present_v). Rotary at positions
    P..P+S-1 when cos/sin are given; causal softmax per query (scores stored
    float32, max / exp / sum in double, as the reference), then scores . V in
    float32 products accumulated in float32 order-insensitively (numpy)."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    b, s, hid = q.shape
    d = hid // num_heads
    group = num_heads // kv_heads
    p = 0 if past_k is None else past_k.shape[2]
    pos = np.broadcast_to(np.arange(p, p + s)[None, :], (b, s))
    if cos is not None:
        q = rotary(q, pos, cos, sin, num_heads, interleaved)
        k = rotary(k, pos, cos, sin, kv_heads, interleaved)
    kn = k.reshape(b, s, kv_heads, d).transpose(0, 2, 1, 3)
    vn = v.reshape(b, s, kv_heads, d).transpose(0, 2, 1, 3)
    pk = kn if past_k is None else np.concatenate([np.asarray(past_k, np.float32), kn], axis=2)
    pv = vn if past_v is None else np.concatenate([np.asarray(past_v, np.float32), vn], axis=2)
    total = p + s
    sc = scale if scale else 1.0 / math.sqrt(d)
    qh = q.reshape(b, s, num_heads, d).transpose(0, 2, 1, 3)  # [B][H][S][D]
    out = np.zeros((b, num_heads, s, d), np.float32)
    for hh in range(num_heads):
        kv = hh // group
        scores = np.matmul(qh[:, hh].astype(np.float64), pk[:, kv].astype(np.float64).transpose(0, 2, 1))
        scores = (scores.astype(np.float32).astype(np.float64) * sc)
        mask = np.arange(total)[None, :] > (p + np.arange(s))[:, None]
        scores = np.where(mask[None], -np.inf, scores)
        mx = scores.max(-1, keepdims=True)
        e = np.exp(scores - mx)
        probs = (e / e.sum(-1, keepdims=True)).astype(np.float32)
        out[:, hh] = np.matmul(probs.astype(np.float64), pv[:, kv].astype(np.float64))
    return out.transpose(0, 2, 1, 3).reshape(b, s, hid), pk, pv


def mha(q, k, v, num_heads, kv_heads=None, mask=None, scale=None, causal=False, bias4d=None):
    """opMultiHeadAttention (lib/src/onnx_ops.dart:2019-2098) / the scale +
    mask + softmax of opFusedSDPA (:2106-2148) per head: q [B][S][H*D], k / v
    [B][T][KVH*D]; mask None or additive [B][T] (a row per batch, broadcast over
    heads and queries); bias4d None or the additive attention bias
    [B][bias_heads][S][T], head h reading bias head h % bias_heads (:2062-2064).
    Scores are a float32 MatMul; scale + bias, max, exp and the sum run in
    double and the probabilities are stored float32; then the float32 MatMul
    with V."""
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    b, s, hid = q.shape
    t = k.shape[1]
    kv_heads = kv_heads or num_heads
    d = hid // num_heads
    group = num_heads // kv_heads
    sc = scale if scale else 1.0 / math.sqrt(d)
    qh = q.reshape(b, s, num_heads, d).transpose(0, 2, 1, 3)
    kh = k.reshape(b, t, kv_heads, d).transpose(0, 2, 1, 3)
    vh = v.reshape(b, t, kv_heads, d).transpose(0, 2, 1, 3)
    out = np.zeros((b, num_heads, s, d), np.float32)
    for hh in range(num_heads):
        kv = hh // group
        scores = np.matmul(qh[:, hh].astype(np.float64), kh[:, kv].astype(np.float64).transpose(0, 2, 1))
        val = scores.astype(np.float32).astype(np.float64) * sc
        if mask is not None:
            val = val + np.asarray(mask, np.float32).astype(np.float64).reshape(b, 1, t)
        if bias4d is not None:
            bb = np.asarray(bias4d, np.float32)
            val = val + bb[:, hh % bb.shape[1]].astype(np.float64)
        val = val.astype(np.float32).astype(np.float64)  # the scores row is stored float32
        if causal:
            val = np.where(np.arange(t)[None, None, :] > np.arange(s)[None, :, None], -np.inf, val)
        e = np.exp(val - val.max(-1, keepdims=True))
        probs = (e / e.sum(-1, keepdims=True)).astype(np.float32)
        out[:, hh] = np.matmul(probs.astype(np.float64), vh[:, kv].astype(np.float64))
    return out.transpose(0, 2, 1, 3).reshape(b, s, hid)
