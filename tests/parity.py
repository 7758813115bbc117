"""Tolerances shared by the parity tests.

bf16 outputs and gradients: max-abs error <= 2e-2 after normalising by the
RMS of the reference tensor.  Scalar losses: 1e-3 relative.  fp32 kernels:
the reference GPU test's 1e-5 absolute/relative tolerance (test_kernels.py:78-79).
"""
from __future__ import annotations

import torch

BF16_RMS_TOL = 2e-2
LOSS_REL_TOL = 1e-3
FP32_TOL = 1e-5


def rms_normalised_max_err(actual: torch.Tensor, expected: torch.Tensor) -> float:
    a = actual.detach().to("cpu", torch.float64)
    e = expected.detach().to("cpu", torch.float64)
    assert a.shape == e.shape, (tuple(a.shape), tuple(e.shape))
    assert torch.isfinite(a).all(), "non-finite values in the CUDA result"
    rms = e.pow(2).mean().sqrt().item()
    err = (a - e).abs().max().item()
    return err / rms if rms > 0 else err


def assert_bf16_close(actual, expected, tol: float = BF16_RMS_TOL, what: str = ""):
    err = rms_normalised_max_err(actual, expected)
    assert err <= tol, f"{what}: max|err|/rms = {err:.3e} > {tol:.1e}"


def assert_loss_close(actual, expected, tol: float = LOSS_REL_TOL, what: str = "loss"):
    a = float(actual)
    e = float(expected)
    assert abs(a - e) <= tol * max(abs(e), 1e-12), f"{what}: {a} vs {e} (rel tol {tol})"


def assert_fp32_close(actual, expected, tol: float = FP32_TOL, what: str = ""):
    a = actual.detach().to("cpu", torch.float64)
    e = expected.detach().to("cpu", torch.float64)
    torch.testing.assert_close(a, e, atol=tol, rtol=tol, msg=lambda m: f"{what}: {m}")
