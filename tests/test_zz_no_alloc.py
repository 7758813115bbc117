"""The allocation-free RMSNorm backward entry point gives the same results as
the workspace entry point.

hlm_residual_rms_norm_bwd_noalloc exists for callers that cannot allocate
device memory when they call the operator: hosts that plan every device byte
up front (a fixed-budget serving process, or a framework whose allocator
cannot be re-entered from inside an operator) and code that must not stall
the GPU, because cudaMalloc and cudaFree synchronise the device.  Instead of
a caller-provided workspace it keeps its scratch in a fixed array inside the
library.

The test calls both entry points through the C ABI (ctypes, raw device
pointers) twice in a row with different shapes and dtypes, so a second call
that read anything left in the shared array by the first would show up as a
mismatch.  This file is collected last so that a failure here cannot hide
any other test's result.
"""
from __future__ import annotations

import ctypes

import pytest
import torch

from parity import assert_bf16_close, assert_fp32_close

pytestmark = pytest.mark.gpu

DTYPE_CODE = {torch.float32: 0, torch.bfloat16: 1}


def _inputs(rows, cols, dtype, seed, device):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g).to(dtype).to(device)
    w = (1.0 + 0.02 * torch.randn(cols, generator=g)).to(dtype).to(device)
    gout = torch.randn(rows, cols, generator=g).to(dtype).to(device)
    gnorm = torch.randn(rows, cols, generator=g).to(dtype).to(device)
    return x, w, gout, gnorm


def _with_workspace(lib, x, w, gout, gnorm, stream):
    rows, cols = x.shape
    gin = torch.empty_like(x)
    gw = torch.empty(cols, dtype=x.dtype, device=x.device)
    nbytes = lib.hlm_rms_norm_bwd_workspace_bytes(rows, cols)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    rc = lib.hlm_residual_rms_norm_bwd(x.data_ptr(), w.data_ptr(), gout.data_ptr(), gnorm.data_ptr(),
                                       gin.data_ptr(), gw.data_ptr(), ws.data_ptr(), nbytes, rows, cols,
                                       ctypes.c_float(1e-6), DTYPE_CODE[x.dtype], stream)
    assert rc == 0, rc
    return gin, gw


def _no_alloc(lib, x, w, gout, gnorm, stream):
    rows, cols = x.shape
    gin = torch.empty_like(x)
    gw = torch.empty(cols, dtype=x.dtype, device=x.device)
    rc = lib.hlm_residual_rms_norm_bwd_noalloc(x.data_ptr(), w.data_ptr(), gout.data_ptr(),
                                               gnorm.data_ptr(), gin.data_ptr(), gw.data_ptr(), rows,
                                               cols, ctypes.c_float(1e-6), DTYPE_CODE[x.dtype], stream)
    assert rc == 0, rc
    return gin, gw


def test_no_alloc_matches_workspace_entry_point(cuda_device):
    from hackable_lm_b200 import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    _lib.clear_device_error(stream)
    cases = [(4096, 1024, torch.bfloat16, 1), (37, 384, torch.float32, 2)]
    for rows, cols, dtype, seed in cases:  # two calls in a row, different shapes
        x, w, gout, gnorm = _inputs(rows, cols, dtype, seed, cuda_device)
        ref_gin, ref_gw = _with_workspace(lib, x, w, gout, gnorm, stream)
        gin, gw = _no_alloc(lib, x, w, gout, gnorm, stream)
        torch.cuda.synchronize()
        if dtype == torch.float32:
            assert_fp32_close(gin, ref_gin, what="grad_in")
            assert_fp32_close(gw, ref_gw, what="grad_weight")
        else:
            assert_bf16_close(gin, ref_gin, what="grad_in")
            assert_bf16_close(gw, ref_gw, what="grad_weight")
    assert _lib.device_error(stream) == 0


def test_no_alloc_scalar_path_and_empty_rows(cuda_device):
    """cols = 383 (not a multiple of the 16-byte vector) takes the scalar kernel;
    rows = 0 must give grad_weight == 0 even though the shared array still holds the
    previous call's partial sums."""
    from hackable_lm_b200 import _lib

    lib = _lib.load()
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    x, w, gout, gnorm = _inputs(500, 383, torch.bfloat16, 4, cuda_device)
    ref_gin, ref_gw = _with_workspace(lib, x, w, gout, gnorm, stream)
    gin, gw = _no_alloc(lib, x, w, gout, gnorm, stream)
    torch.cuda.synchronize()
    assert_bf16_close(gin, ref_gin, what="grad_in (scalar path)")
    assert_bf16_close(gw, ref_gw, what="grad_weight (scalar path)")
    empty = torch.empty(0, 383, dtype=torch.bfloat16, device=cuda_device)
    gw0 = torch.full((383,), 7.0, dtype=torch.bfloat16, device=cuda_device)
    rc = lib.hlm_residual_rms_norm_bwd_noalloc(empty.data_ptr(), w.data_ptr(), None, empty.data_ptr(),
                                               empty.data_ptr(), gw0.data_ptr(), 0, 383, ctypes.c_float(1e-6),
                                               1, stream)
    assert rc == 0, rc
    torch.cuda.synchronize()
    assert torch.count_nonzero(gw0) == 0


def test_no_alloc_rejects_too_many_columns(cuda_device):
    from hackable_lm_b200 import _lib

    lib = _lib.load()
    x, w, gout, gnorm = _inputs(8, 2048, torch.bfloat16, 3, cuda_device)
    gin = torch.empty_like(x)
    gw = torch.empty(2048, dtype=x.dtype, device=cuda_device)
    rc = lib.hlm_residual_rms_norm_bwd_noalloc(x.data_ptr(), w.data_ptr(), gout.data_ptr(), gnorm.data_ptr(),
                                               gin.data_ptr(), gw.data_ptr(), 8, 2048, ctypes.c_float(1e-6),
                                               1, torch.cuda.current_stream(cuda_device).cuda_stream)
    assert rc == -2  # HLM_ERR_UNSUPPORTED: beyond HLM_NOALLOC_RMS_MAX_COLS
