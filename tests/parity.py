"""Parity rules shared by the tests.

Attention (the three-way rule). ggml's CPU flash attention is itself far from exact for f16 V (it
accumulates V*softmax in fp16, ops.cpp:8992-9007), so "within 2e-3 of ggml" is stated against the exact
value computed in f64 on the same cache contents, with Q rounded the way both implementations round it
(f16 for an f16 cache, q8_0 for a q8_0 cache, ops.cpp:8960):

    e_gpu = max|gpu - f64| / max|f64|                <= ATTN_TOL (2e-3)
    e_cpu = max|ggml - f64| / max|f64|                  (the oracle's own error, reported)
    max|gpu - ggml| / max|f64|                       <= e_cpu + ATTN_TOL

DeltaNet: state and output within DELTANET_TOL (1e-3) of f64, max error relative to max|f64|.
Rollback and cache writes: bit-exact.
"""
from __future__ import annotations

import numpy as np

ATTN_TOL = 2e-3
DELTANET_TOL = 1e-3


def rel_err(a, b, den=None) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.abs(b).max() if den is None else den
    if den == 0:
        return float(np.abs(a - b).max())
    return float(np.abs(a - b).max() / den)


def check_attention(gpu, exact, ggml=None, tol=ATTN_TOL):
    """Asserts the three-way rule; returns (e_gpu, e_cpu, e_gpu_vs_ggml)."""
    gpu = np.asarray(gpu, dtype=np.float64)
    exact = np.asarray(exact, dtype=np.float64)
    assert np.isfinite(gpu).all(), "non-finite values in the GPU output"
    den = np.abs(exact).max()
    e_gpu = rel_err(gpu, exact, den)
    assert e_gpu <= tol, f"GPU vs f64: {e_gpu:.3e} > {tol:.1e}"
    e_cpu = e_vs = None
    if ggml is not None:
        e_cpu = rel_err(ggml, exact, den)
        e_vs = rel_err(gpu, ggml, den)
        assert e_vs <= e_cpu + tol, f"GPU vs ggml: {e_vs:.3e} > e_cpu {e_cpu:.3e} + {tol:.1e}"
    return e_gpu, e_cpu, e_vs
