"""Shared pytest configuration: the `gpu` marker and golden-vector helpers."""
import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN_DIR = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the CUDA kernels")


def golden_cases(prefix=""):
    names = sorted(f[:-5] for f in os.listdir(GOLDEN_DIR) if f.endswith(".json"))
    return [n for n in names if n.startswith(prefix)]


def load_golden(name):
    with open(os.path.join(GOLDEN_DIR, name + ".json")) as f:
        g = json.load(f)

    def arr(t):
        if t is None:
            return None
        t = t["tensor"] if "tensor" in t else t
        return np.array(t["data"], dtype=np.dtype(t["dtype"])).reshape(t["shape"])

    g["arrays"] = [None if i is None else arr(i) for i in g["inputs"]]
    g["expected_arrays"] = {k: arr(v) for k, v in g["expected"].items()}
    return g


def assert_fixture_close(have, want, what=""):
    """The reference's fixture tolerance (test/fixture_parity_test.dart:21, 65-108):
    ints exact; floats max|d| <= max(2e-5, 2e-5*max|ref|) and cosine > 0.999999."""
    have = np.asarray(have)
    want = np.asarray(want)
    assert list(have.shape) == list(want.shape), f"{what}: shape {have.shape} != {want.shape}"
    if want.dtype.kind in "iu":
        np.testing.assert_array_equal(have.astype(np.int64), want.astype(np.int64), err_msg=what)
        return
    w = want.astype(np.float64).ravel()
    h = have.astype(np.float64).ravel()
    max_abs = float(np.max(np.abs(w - h))) if w.size else 0.0
    max_mag = float(np.max(np.abs(w))) if w.size else 0.0
    tol = max(2e-5, 2e-5 * max_mag)
    assert max_abs <= tol, f"{what}: max|d|={max_abs} > {tol}"
    nw, nh = float(np.dot(w, w)), float(np.dot(h, h))
    if nw > 0 and nh > 0:
        cos = float(np.dot(w, h)) / (np.sqrt(nw) * np.sqrt(nh))
        assert cos > 0.999999, f"{what}: cosine={cos}"


def assert_fast_close(have, want, what="", max_rel=1e-3, min_cos=0.99999):
    """Fast (tensor-core) mode tolerance from the path's contract: max relative
    error <= 1e-3, measured as max|d| / max|ref|, and cosine >= 0.99999."""
    have = np.asarray(have, np.float64).ravel()
    want = np.asarray(want, np.float64).ravel()
    assert have.shape == want.shape, what
    if want.size == 0:
        return
    scale = float(np.max(np.abs(want)))
    err = float(np.max(np.abs(have - want)))
    rel = err / scale if scale > 0 else err
    assert np.all(np.isfinite(have)), f"{what}: non-finite output"
    assert rel <= max_rel, f"{what}: max rel err {rel:.3e} > {max_rel}"
    nw, nh = float(np.dot(want, want)), float(np.dot(have, have))
    if nw > 0 and nh > 0:
        cos = float(np.dot(want, have)) / np.sqrt(nw * nh)
        assert cos >= min_cos, f"{what}: cosine {cos} < {min_cos}"
