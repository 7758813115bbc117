"""ctypes binding of libhlm_b200.so (the C ABI declared in include/hlm_b200.h).

The shared library is built in-tree by ``python -m hackable_lm_b200.build``.
There is no fallback: if the library is missing or fails to load, every
operator raises, so a GPU run can never silently take a different path.
"""
from __future__ import annotations

import ctypes
import os
import threading
from ctypes import POINTER, c_char_p, c_float, c_int, c_int64, c_size_t, c_uint64, c_void_p
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libhlm_b200.so"

HLM_OK = 0
HLM_F32, HLM_BF16, HLM_F16 = 0, 1, 2

_P = c_void_p
_I64 = c_int64
_I64P = POINTER(c_int64)

# name -> (argtypes, restype); mirrors include/hlm_b200.h one to one.
SIGNATURES: dict[str, tuple[list, object]] = {
    "hlm_version": ([], c_int),
    "hlm_strerror": ([c_int], c_char_p),
    "hlm_device_error_get": ([POINTER(c_int), _P], c_int),
    "hlm_device_error_clear": ([_P], c_int),
    "hlm_selftest_bounded_wait": ([_I64, c_int, _P], c_int),
    "hlm_launch_count": ([], c_uint64),
    "hlm_profile_begin": ([c_int, POINTER(c_void_p), POINTER(c_void_p), c_int], c_int),
    "hlm_profile_end": ([c_int, POINTER(c_int)], c_int),
    "hlm_swiglu_fwd": ([_P, _P, _I64, _I64, c_int, _P], c_int),
    "hlm_swiglu_bwd": ([_P, _P, _P, _I64, _I64, c_int, _P], c_int),
    "hlm_residual_rms_norm_fwd": ([_P, _P, _P, _P, _P, _I64, _I64, c_float, c_int, _P], c_int),
    "hlm_residual_rms_norm_bwd": (
        [_P, _P, _P, _P, _P, _P, _P, c_size_t, _I64, _I64, c_float, c_int, _P], c_int),
    "hlm_rms_norm_bwd_workspace_bytes": ([_I64, _I64], c_size_t),
    "hlm_residual_rms_norm_bwd_noalloc": (
        [_P, _P, _P, _P, _P, _P, _I64, _I64, c_float, c_int, _P], c_int),
    "hlm_qk_norm_rope_fwd": (
        [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64P, _I64P, _I64, c_int,
         c_float, c_int, _P], c_int),
    "hlm_qk_norm_rope_bwd": (
        [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64P, _I64P, _I64,
         c_int, c_float, c_int, _P], c_int),
    "hlm_qkv_rope_fwd": (
        [_P, _P, _P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _I64, _I64, c_int,
         c_float, _P], c_int),
    "hlm_qkv_rope_bwd": (
        [_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, _I64, _I64, _I64, _I64,
         _I64, _I64, _I64, _I64, c_int, c_float, _P], c_int),
    "hlm_qkv_rope_bwd_workspace_bytes": ([_I64, _I64, _I64, _I64, _I64, _I64], c_size_t),
    "hlm_lm_head_ce": (
        [_P, _P, _P, _P, _P, _P, _P, c_size_t, _I64, _I64, _I64, _I64, _I64, _P], c_int),
    "hlm_lm_head_ce_workspace_bytes": ([_I64, _I64, _I64, _I64], c_size_t),
    "hlm_scale_by_device_scalar": ([_P, _P, _I64, c_int, _P], c_int),
    "hlm_gate_up_swiglu_fwd": ([_P, _P, _P, _P, _I64, _I64, _I64, _P], c_int),
    "hlm_swiglu_down_bwd": ([_P, _P, _P, _P, _I64, _I64, _I64, _P], c_int),
    "hlm_proj_residual_rms_norm_fwd": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, c_float, _P], c_int),
    "hlm_attention_fwd": ([_P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, c_float, _P], c_int),
    "hlm_attention_bwd_workspace_bytes": ([_I64, _I64, _I64, _I64], c_size_t),
    "hlm_attention_bwd": ([_P, _P, _P, _P, _P, _P, _P, _P, _P, _P, c_size_t, _I64, _I64, _I64, _I64, _I64, _I64,
                           c_float, _P], c_int),
    "hlm_gemm_bf16": (
        [_P, _P, _P, _I64, _I64, _I64, c_int, c_int, _I64, _I64, _I64, c_int, c_int, _P], c_int),
}

_lib = None
_lock = threading.Lock()


class HlmError(RuntimeError):
    """A libhlm_b200 entry point returned a non-zero status."""


def load() -> ctypes.CDLL:
    """Load libhlm_b200.so once and attach the C signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = Path(os.environ.get("HLM_B200_LIB", str(LIB_PATH)))
        if not path.exists():
            raise HlmError(
                f"hackable_lm_b200 CUDA library not found at {path}; "
                "build it with `python -m hackable_lm_b200.build`"
            )
        # Load after torch so the library binds to the process's CUDA runtime.
        import torch  # noqa: F401

        lib = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
        for name, (argtypes, restype) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != HLM_OK:
        msg = load().hlm_strerror(rc)
        raise HlmError(f"{what} failed: {msg.decode() if msg else rc} (code {rc})")


def device_error(stream: int = 0) -> int:
    """Synchronously read the device error word (0 = no kernel reported a problem)."""
    out = c_int(0)
    check(load().hlm_device_error_get(ctypes.byref(out), c_void_p(stream)), "hlm_device_error_get")
    return out.value


def clear_device_error(stream: int = 0) -> None:
    check(load().hlm_device_error_clear(c_void_p(stream)), "hlm_device_error_clear")


# Device error word codes (HLM_DEVERR_* in include/hlm_b200.h).
DEVERR_NAMES = {
    0: "none", 1: "timeout: MMA issuer waiting for a TMA stage",
    2: "timeout: producer waiting for a free stage", 3: "timeout: epilogue waiting for an accumulator",
    4: "timeout: MMA issuer waiting for the epilogue", 5: "timeout: teardown drain of TMA copies",
    6: "unexpected tensor-memory address", 7: "self-test wait ran out (expected)",
    8: "timeout: epilogue waiting for its input tile",
    9: "timeout: epilogue waiting for its cluster peers' row sums",
}
DEVERR_SELFTEST_TIMEOUT = 7


def selftest_bounded_wait(limit_us: int, scope: int = 0, stream: int = 0) -> None:
    """Launch the bounded-wait self-test (a wait on an mbarrier nothing arrives at,
    limited to limit_us); it records DEVERR_SELFTEST_TIMEOUT in the device error word."""
    check(load().hlm_selftest_bounded_wait(int(limit_us), int(scope), c_void_p(stream)),
          "hlm_selftest_bounded_wait")


# Kernel ids of hlm_profile_begin (include/hlm_b200.h).
KERNEL_IDS = {
    "lm_logits": 1, "lm_dlogits": 2, "lm_dx": 3, "lm_dw": 4, "qkv_fwd": 5, "qkv_bwd_norm": 6,
    "qkv_dx": 7, "qkv_dw": 8, "swiglu_fwd": 9, "swiglu_bwd": 10, "rmsnorm_fwd": 11,
    "rmsnorm_bwd": 12, "qk_rope_fwd": 13, "qk_rope_bwd": 14, "gemm": 15, "gate_up": 16,
    "swiglu_down_bwd": 17, "proj_norm": 18, "attn_fwd": 19, "attn_bwd": 20,
}


def launch_count() -> int:
    """Kernels launched by libhlm_b200 in this process so far."""
    return int(load().hlm_launch_count())


class KernelTimer:
    """Time every launch of one library kernel with CUDA events recorded by the
    library itself on the launching stream (hlm_profile_begin/end)."""

    def __init__(self, kernel: str, capacity: int):
        import torch

        self.kid = KERNEL_IDS[kernel]
        self.capacity = capacity
        self.starts = [torch.cuda.Event(enable_timing=True) for _ in range(capacity)]
        self.stops = [torch.cuda.Event(enable_timing=True) for _ in range(capacity)]
        for ev in self.starts + self.stops:
            ev.record()  # materialise the underlying cudaEvent_t
        self._a = (c_void_p * capacity)(*[ev.cuda_event for ev in self.starts])
        self._b = (c_void_p * capacity)(*[ev.cuda_event for ev in self.stops])
        self.launches = 0

    def __enter__(self):
        check(load().hlm_profile_begin(self.kid, self._a, self._b, self.capacity), "hlm_profile_begin")
        return self

    def __exit__(self, *exc):
        n = c_int(0)
        check(load().hlm_profile_end(self.kid, ctypes.byref(n)), "hlm_profile_end")
        self.launches = n.value
        return False

    def times_ms(self) -> list[float]:
        import torch

        torch.cuda.synchronize()
        k = min(self.launches, self.capacity)
        return [self.starts[i].elapsed_time(self.stops[i]) for i in range(k)]


def int64_array(values) -> ctypes.Array:
    arr = (c_int64 * len(values))(*[int(v) for v in values])
    return arr
