"""The config-4 / config-5 chain compositions of oracle/chains.py applied to
the drivers' kept host weights — TEST INFRASTRUCTURE ONLY."""
from __future__ import annotations

import numpy as np

from oracle import chains

THREADS = chains.THREADS


class NbitsWeights(chains.DequantCache):
    """Exactly dequantized MatMulNBits weights of a decoder's kept host weights."""

    def __init__(self, dec):
        super().__init__(dec.cfg, dec.host)


def ref_decoder(dec, ids, past, strict=True, weights=None):
    """chains.decoder_forward on the decoder `dec` (kept host weights)."""
    return chains.decoder_forward(dec.cfg, dec.host, dec.cap, ids, past, strict=strict, weights=weights)


def ref_bert(enc, ids, mask01):
    """chains.bert_forward on the encoder `enc` (kept host weights)."""
    return chains.bert_forward(enc.cfg, enc.host, ids, mask01)


def rel_cos(have, want):
    """(max|d| / max|ref|, cosine) in float64."""
    h = np.asarray(have, np.float64).ravel()
    w = np.asarray(want, np.float64).ravel()
    rel = float(np.max(np.abs(h - w)) / max(float(np.max(np.abs(w))), 1e-30))
    cos = float(np.dot(h, w) / np.sqrt(np.dot(h, h) * np.dot(w, w)))
    return rel, cos
