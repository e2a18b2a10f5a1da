"""Parity metrics and tolerances shared by the GPU tests, smoke() and bench.

``metrics`` restates the reference's own accuracy report
(tools/test_seedvr2_dit_ncnn.py:40-62: max_abs, mean_abs, rmse, nrmse vs the
reference RMS, cosine, finite).

Tolerances (per attention layer, against the oracle on identical inputs):
  * max_abs <= 2e-3 and cosine >= 0.9999 (the north-star gate);
  * for the bf16-rounded output mode the reference itself rounds every window
    output to bf16 (seedvr2_dit_block.cpp:1074); an fp32-accumulating tensor
    core result that lands on the other side of a rounding boundary differs
    by one bf16 ulp, which exceeds 2e-3 when |out| >= 0.5. That mode is
    therefore gated elementwise at max(2e-3, one bf16 ulp of the reference
    value), plus the same cosine; fp16 outputs use the plain 2e-3 gate.
"""
from __future__ import annotations

import numpy as np

MAX_ABS = 2e-3
COSINE = 0.9999


def metrics(actual, expected) -> dict:
    a = np.asarray(actual, np.float64).reshape(-1)
    e = np.asarray(expected, np.float64).reshape(-1)
    d = a - e
    rmse = float(np.sqrt(np.mean(d * d)))
    ref_rms = max(float(np.sqrt(np.mean(e * e))), 1e-12)
    den = max(float(np.sqrt(np.sum(a * a) * np.sum(e * e))), 1e-12)
    return {
        "finite": bool(np.isfinite(a).all() and np.isfinite(e).all()),
        "max_abs": float(np.abs(d).max()),
        "mean_abs": float(np.abs(d).mean()),
        "rmse": rmse,
        "nrmse": rmse / ref_rms,
        "cosine": float(np.sum(a * e) / den),
        "exact_frac": float(np.mean(d == 0)),
    }


def bf16_ulp(x) -> np.ndarray:
    """Spacing of bf16 values at |x| (2^(exponent - 7))."""
    ax = np.abs(np.asarray(x, np.float32))
    e = np.floor(np.log2(np.maximum(ax, np.float32(2.0 ** -126))))
    return np.exp2(e - 7).astype(np.float64)


def check(actual, expected, bf16_rounded: bool, what: str = "") -> dict:
    m = metrics(actual, expected)
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    tol = np.maximum(MAX_ABS, bf16_ulp(e)) if bf16_rounded else MAX_ABS
    bad = np.abs(a - e) > tol
    assert m["finite"], f"{what}: non-finite values {m}"
    assert not bad.any(), f"{what}: {int(bad.sum())} elements beyond tolerance; {m}"
    assert m["cosine"] >= COSINE, f"{what}: cosine {m['cosine']} < {COSINE}; {m}"
    return m
