"""Tolerances shared by the parity tests.

bf16 outputs and gradients: every element must satisfy
    |actual - expected| <= 2e-2 * (rms(expected) + |expected|)
i.e. the "max-abs error <= 2e-2 after normalising by the reference RMS" bar,
widened by 2e-2 relative for elements far above the RMS.  The widening is
needed because bf16 itself cannot meet the pure RMS-normalised bar on
heavy-tailed tensors: a correctly rounded bf16 value carries up to 2^-9 of
its own magnitude, so a SwiGLU output whose max is 20x its RMS already sits
at 4% of the RMS after exact rounding.  2e-2 relative is ~2.5 bf16 ulps.

Scalar losses: 1e-3 relative.  fp32 kernels: 1e-5 absolute and relative,
the reference GPU test's tolerance (tests/test_kernels.py:78-79 upstream).
"""
from __future__ import annotations

import json
import os

import torch

BF16_TOL = 2e-2
LOSS_REL_TOL = 1e-3
FP32_TOL = 1e-5


def _pair(actual, expected):
    a = actual.detach().to("cpu", torch.float64)
    e = expected.detach().to("cpu", torch.float64)
    assert a.shape == e.shape, (tuple(a.shape), tuple(e.shape))
    assert torch.isfinite(a).all(), "non-finite values in the CUDA result"
    return a, e


def rms_normalised_max_err(actual, expected) -> float:
    """max|a - e| / rms(e) (reported alongside the bf16-aware check)."""
    a, e = _pair(actual, expected)
    rms = e.pow(2).mean().sqrt().item()
    err = (a - e).abs().max().item()
    return err / rms if rms > 0 else err


def bf16_err(actual, expected) -> float:
    """max_i |a_i - e_i| / (rms(e) + |e_i|)."""
    a, e = _pair(actual, expected)
    rms = e.pow(2).mean().sqrt()
    denom = rms + e.abs()
    denom = torch.where(denom > 0, denom, torch.ones_like(denom))
    return ((a - e).abs() / denom).max().item()


def record(what: str, **metrics) -> None:
    """Append one JSON line {test, what, metrics} to $HLM_PARITY_LOG when it is set, so a
    GPU run leaves a table of every comparison's measured error (not just pass/fail)."""
    path = os.environ.get("HLM_PARITY_LOG")
    if not path:
        return
    test = os.environ.get("PYTEST_CURRENT_TEST", "").split(" ")[0]
    with open(path, "a") as f:
        f.write(json.dumps({"test": test, "what": what, **metrics}) + "\n")


def assert_bf16_close(actual, expected, tol: float = BF16_TOL, what: str = ""):
    err = bf16_err(actual, expected)
    strict = rms_normalised_max_err(actual, expected)
    record(what, bf16_err=err, max_err_over_rms=strict, tol=tol)
    assert err <= tol, (f"{what}: max|err|/(rms+|ref|) = {err:.3e} > {tol:.1e} "
                        f"(max|err|/rms = {strict:.3e})")


def assert_loss_close(actual, expected, tol: float = LOSS_REL_TOL, what: str = "loss"):
    a = float(actual)
    e = float(expected)
    rel = abs(a - e) / max(abs(e), 1e-12)
    record(what, loss_rel_err=rel, tol=tol)
    assert rel <= tol, f"{what}: {a} vs {e} (rel err {rel:.3e} > tol {tol})"


def assert_fp32_close(actual, expected, tol: float = FP32_TOL, what: str = ""):
    a, e = _pair(actual, expected)
    torch.testing.assert_close(a, e, atol=tol, rtol=tol, msg=lambda m: f"{what}: {m}")
