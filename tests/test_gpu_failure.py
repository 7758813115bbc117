"""Failure detection on the GPU without a fault: a bounded mbarrier wait that
nothing satisfies runs out after its limit, the kernel records its code in the
device error word and returns, and the context stays usable (a GEMM launched
afterwards is correct and reports no error)."""
from __future__ import annotations

import time

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("scope", [0, 1])
def test_bounded_wait_runs_out_and_context_survives(scope, cuda_device):
    from hackable_lm_b200 import _lib, ops

    torch.cuda.synchronize()
    _lib.clear_device_error()
    assert _lib.device_error() == 0
    t0 = time.perf_counter()
    _lib.selftest_bounded_wait(20_000, scope)  # 20 ms limit
    code = _lib.device_error()  # synchronises
    elapsed = time.perf_counter() - t0
    assert code == _lib.DEVERR_SELFTEST_TIMEOUT, _lib.DEVERR_NAMES.get(code, code)
    assert 0.015 < elapsed < 5.0  # the wait lasted about its limit, and ended
    _lib.clear_device_error()

    g = torch.Generator().manual_seed(scope)
    a = torch.randn(512, 256, generator=g).to(torch.bfloat16)
    b = torch.randn(384, 256, generator=g).to(torch.bfloat16)
    d = ops.gemm(a.to(cuda_device), b.to(cuda_device))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    ref = a.float() @ b.float().t()
    err = (d.float().cpu() - ref).abs().max() / ref.abs().max()
    assert err < 1e-2
