"""Comparison helpers of the GPU parity tests.

Two bars:
  * exact: the decode paths (tile GEMV, persistent kernel, attention, the
    int8 tensor-core prefill) follow the arithmetic convention the CPU oracle
    shares, so their outputs must equal the oracle's bit for bit
    (max|delta| == 0).
  * tolerance: the fp16 tensor-core prefill of F16 models sums the exact
    products in fp32 over the whole row, so it (and any step that reads the
    K/V it cached) is held to the parity contract's bound
    max|delta| <= 1e-2 * std(logits).
"""
from __future__ import annotations

import numpy as np

LOGIT_TOL = 1e-2


def assert_exact(got: np.ndarray, want: np.ndarray, what: str) -> None:
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    assert np.isfinite(got).all(), f"{what}: non-finite values"
    if not np.array_equal(got, want):
        d = np.abs(got.astype(np.float64) - want.astype(np.float64))
        raise AssertionError(f"{what}: not bit-exact, {int((d > 0).sum())} of {d.size} differ, "
                             f"max|delta| {d.max():.3e} ({d.max() / max(float(want.std()), 1e-30):.2e} std)")


def assert_close(got: np.ndarray, want: np.ndarray, what: str) -> None:
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    assert np.isfinite(got).all(), f"{what}: non-finite values"
    err = float(np.abs(got - want).max())
    bound = LOGIT_TOL * float(want.std())
    assert err <= bound, f"{what}: max|delta| {err:.3e} > {bound:.3e}"
