"""The tcgen05 GEMM core against a PyTorch fp32 matmul of the same bf16 operands,
for every operand-major combination and for shapes that are not tile multiples."""
from __future__ import annotations

import pytest
import torch

from parity import assert_bf16_close

pytestmark = pytest.mark.gpu


def _operands(M, N, K, a_mn, b_mn, device, seed=0):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(M, K, generator=g).to(torch.bfloat16)
    b = torch.randn(N, K, generator=g).to(torch.bfloat16)
    a_store = a.t().contiguous() if a_mn else a
    b_store = b.t().contiguous() if b_mn else b
    return a, b, a_store.to(device), b_store.to(device)


@pytest.mark.parametrize("a_mn,b_mn", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 768), (200, 136, 136), (1000, 768, 2304),
                                   (64, 64, 64), (704, 1152, 8192)])
def test_gemm_layouts(M, N, K, a_mn, b_mn, cuda_device):
    from hackable_lm_b200 import _lib, ops

    _lib.clear_device_error()
    a, b, a_s, b_s = _operands(M, N, K, a_mn, b_mn, cuda_device)
    ref = a.to(cuda_device).float() @ b.to(cuda_device).float().t()
    out32 = ops.gemm(a_s, b_s, a_mn_major=a_mn, b_mn_major=b_mn, out_dtype=torch.float32)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    err = (out32 - ref).abs().max().item() / ref.pow(2).mean().sqrt().item()
    assert err < 1e-3, f"fp32-out GEMM error {err:.2e}"
    out16 = ops.gemm(a_s, b_s, a_mn_major=a_mn, b_mn_major=b_mn, out_dtype=torch.bfloat16)
    assert_bf16_close(out16, ref, what="bf16-out GEMM")


def test_gemm_accumulate(cuda_device):
    from hackable_lm_b200 import ops

    a, b, a_s, b_s = _operands(256, 256, 128, False, False, cuda_device)
    base = torch.randn(256, 256, device=cuda_device)
    out = base.clone()
    ops.gemm(a_s, b_s, out=out, accumulate=True)
    ref = base + a.to(cuda_device).float() @ b.to(cuda_device).float().t()
    assert (out - ref).abs().max().item() < 1e-2


def test_gemm_large_k(cuda_device):
    """K = 32768: the LM-head dX/dW reduction depth."""
    from hackable_lm_b200 import ops

    a, b, a_s, b_s = _operands(256, 768, 32768, False, True, cuda_device)
    ref = a.to(cuda_device).float() @ b.to(cuda_device).float().t()
    out = ops.gemm(a_s, b_s, b_mn_major=True, out_dtype=torch.float32)
    err = (out - ref).abs().max().item() / ref.pow(2).mean().sqrt().item()
    assert err < 1e-3
