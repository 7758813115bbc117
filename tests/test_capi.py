"""The C-ABI library builds, loads and exports exactly what include/hlm_b200.h declares.

No compute call is made here (these run on machines without a GPU): only
symbol lookups, error strings, workspace-size arithmetic and argument
validation that returns before touching the device.
"""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from hackable_lm_b200 import _lib

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "hlm_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hlm_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    if not _lib.LIB_PATH.exists():
        from hackable_lm_b200 import build

        build.build()
    return _lib.load()


def test_header_and_binding_table_agree():
    assert declared_functions() == sorted(_lib.SIGNATURES)


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(str(_lib.LIB_PATH))
    for name in declared_functions():
        assert hasattr(raw, name), f"{name} is declared in hlm_b200.h but not exported"


def test_version_and_error_strings(lib):
    assert lib.hlm_version() >= 100
    assert lib.hlm_strerror(0) == b"ok"
    for code in (-1, -2, -3, -4, -5):
        assert lib.hlm_strerror(code) not in (b"ok", b"unknown error code")
    assert lib.hlm_strerror(-99) == b"unknown error code"


def test_invalid_arguments_are_rejected_before_any_launch(lib):
    # negative sizes / null pointers return HLM_ERR_INVALID_ARG without a CUDA call
    assert lib.hlm_swiglu_fwd(None, None, -1, 4, _lib.HLM_BF16, None) == -1
    assert lib.hlm_swiglu_fwd(None, None, 4, 4, _lib.HLM_BF16, None) == -1
    assert lib.hlm_swiglu_bwd(None, None, None, 4, -4, _lib.HLM_BF16, None) == -1
    assert lib.hlm_residual_rms_norm_fwd(None, None, None, None, None, 4, 8, 1e-6, 1, None) == -1
    assert lib.hlm_lm_head_ce(None, None, None, None, None, None, None, 0, 0, 8, 8, -1, 0, None) == -1
    assert lib.hlm_gemm_bf16(None, None, None, -1, 8, 8, 0, 0, 8, 8, 8, 1, 0, None) == -1
    # empty problems are no-ops
    assert lib.hlm_swiglu_fwd(None, None, 0, 4, _lib.HLM_BF16, None) == 0
    assert lib.hlm_gemm_bf16(None, None, None, 0, 8, 8, 0, 0, 8, 8, 8, 1, 0, None) == 0
    # unsupported dtype code
    assert lib.hlm_swiglu_fwd(ctypes.c_void_p(16), ctypes.c_void_p(16), 4, 4, 7, None) == -2
    # fused QKV only supports head_dim 128
    assert lib.hlm_qkv_rope_fwd(*([None] * 8), 1, 8, 64, 1, 1, 64, 32, 32, 1, 1e-6, None) == -2
    # fused gate_up / down-backward GEMMs: bad sizes, null pointers, unsupported widths
    V16 = ctypes.c_void_p(16)
    assert lib.hlm_gate_up_swiglu_fwd(None, None, None, None, -1, 64, 128, None) == -1
    assert lib.hlm_gate_up_swiglu_fwd(None, None, None, None, 256, 64, 128, None) == -1
    assert lib.hlm_gate_up_swiglu_fwd(V16, V16, V16, V16, 256, 96, 128, None) == -2   # C % 64
    assert lib.hlm_gate_up_swiglu_fwd(V16, V16, V16, V16, 256, 64, 96, None) == -2    # H % 128
    assert lib.hlm_gate_up_swiglu_fwd(None, None, None, None, 0, 64, 128, None) == 0  # empty
    assert lib.hlm_swiglu_down_bwd(None, None, None, None, -1, 64, 256, None) == -1
    assert lib.hlm_swiglu_down_bwd(None, None, None, None, 256, 64, 256, None) == -1
    assert lib.hlm_swiglu_down_bwd(V16, V16, V16, V16, 256, 64, 128, None) == -2      # H % 256
    assert lib.hlm_swiglu_down_bwd(V16, V16, V16, V16, 256, 100, 256, None) == -2     # C % 64
    assert lib.hlm_swiglu_down_bwd(None, None, None, None, 0, 64, 256, None) == 0     # empty
    # bounded-wait self-test: limit outside 1 us .. 1 s, or an unknown scope
    assert lib.hlm_selftest_bounded_wait(0, 0, None) == -1
    assert lib.hlm_selftest_bounded_wait(2_000_000, 0, None) == -1
    assert lib.hlm_selftest_bounded_wait(1000, 2, None) == -1


def test_workspace_queries(lib):
    n, c, v = 32768, 768, 32768
    full = lib.hlm_lm_head_ce_workspace_bytes(n, c, v, 0)
    # whole-batch chunk: at least the bf16 logits of all rows
    assert full >= n * v * 2
    small = lib.hlm_lm_head_ce_workspace_bytes(n, c, v, 4096)
    assert 4096 * v * 2 <= small < full
    assert lib.hlm_rms_norm_bwd_workspace_bytes(1024, 384) > 0
    assert lib.hlm_qkv_rope_bwd_workspace_bytes(16, 2048, 768, 6, 6, 128) >= 2 * 16 * 2048 * 768 * 2


def test_device_error_codes_match_header():
    """The Python names of the device error codes cover exactly HLM_DEVERR_* of the header."""
    text = HEADER.read_text()
    codes = {int(v) for v in re.findall(r"#define HLM_DEVERR_[A-Z_]+ (\d+)", text)}
    assert codes == set(_lib.DEVERR_NAMES)
    assert _lib.DEVERR_SELFTEST_TIMEOUT == int(re.search(r"#define HLM_DEVERR_SELFTEST_TIMEOUT (\d+)", text).group(1))
