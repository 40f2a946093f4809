"""Tolerances of the parity contract, shared by the CPU and GPU tests.

* Integer work (codes, row indices, gathered rows, top-k ids): bit-exact.
* fp32 outputs: within 1e-5 relative -- rtol 1e-5 plus an absolute floor of 1e-5 times the
  reference array's largest magnitude (the reference's own cross-implementation tolerance is
  rtol = atol = 1e-5, ``tests/test_live_export.py:117`` in the reference project).
* bf16 outputs: within 1e-2 relative to the reference array's largest magnitude.
* Codes computed from raw inputs may differ only where the reference logit is within
  ``TAU`` of zero (the reference accepts < 1e-3 sign flips, ``tests/test_live_drafter.py:112``).
"""

from __future__ import annotations

import numpy as np

FP32_RTOL = 1e-5
BF16_TOL = 1e-2
TAU = 1e-4


def assert_fp32_close(got, want, rtol: float = FP32_RTOL, what: str = "") -> None:
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    scale = float(np.max(np.abs(want))) if want.size else 0.0
    np.testing.assert_allclose(got, want, rtol=rtol, atol=rtol * max(scale, 1e-30), err_msg=what)


def assert_bf16_close(got, want, tol: float = BF16_TOL, what: str = "") -> None:
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    scale = float(np.max(np.abs(want))) if want.size else 0.0
    err = float(np.max(np.abs(got - want))) if want.size else 0.0
    assert err <= tol * max(scale, 1e-30), f"{what}: max abs err {err:.3e} > {tol} * {scale:.3e}"


def code_mismatch_ok(got_codes, want_codes, ref_logits, bits: int, tau: float = TAU) -> float:
    """Assert codes agree wherever every reference logit of the route is at least ``tau`` away
    from zero; returns the overall mismatch fraction."""
    got = np.asarray(got_codes).astype(np.int64)
    want = np.asarray(want_codes).astype(np.int64)
    lg = np.asarray(ref_logits, np.float64)
    lg = lg.reshape(*want.shape, bits)
    safe = np.all(np.abs(lg) >= tau, axis=-1)
    bad = (got != want) & safe
    assert not bad.any(), f"{int(bad.sum())} code mismatches away from |logit| < {tau}"
    return float((got != want).mean())
