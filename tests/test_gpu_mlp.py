"""gate_up projection with the SwiGLU activation in the GEMM epilogue, against the
CPU oracle (fp32 GEMM of the same bf16 operands, rounded to bf16 as the
reference's cuBLAS output is, then the oracle SwiGLU), forward and backward."""
from __future__ import annotations

import pytest
import torch

import oracle
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu


def _operands(M, C, H, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, C, generator=g).to(torch.bfloat16)
    w = (torch.randn(2 * H, C, generator=g) * 0.02).to(torch.bfloat16)
    gh = torch.randn(M, H, generator=g).to(torch.bfloat16)
    return x, w, gh


@pytest.mark.parametrize("M,C,H", [(256, 256, 128), (300, 768, 512), (4096, 768, 2048), (1000, 128, 256)])
def test_gate_up_swiglu_vs_oracle(M, C, H, cuda_device):
    from hackable_lm_b200 import _lib, ops

    _lib.clear_device_error()
    x, w, gh = _operands(M, C, H)
    xd = x.to(cuda_device).requires_grad_(True)
    wd = w.to(cuda_device).requires_grad_(True)
    h, gate_up = ops.gate_up_swiglu(xd, wd)
    h.backward(gh.to(cuda_device))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0

    # oracle: the reference's F.linear output (bf16) then its SwiGLU, grads by autograd in fp32
    gu_ref = (x.float() @ w.float().t()).to(torch.bfloat16)
    h_ref = oracle.swiglu(gu_ref)
    assert_bf16_close(gate_up, gu_ref.float(), what="gate_up")
    assert_bf16_close(h, h_ref, what="h")
    xr = x.float().requires_grad_(True)
    wr = w.float().requires_grad_(True)
    gr = xr @ wr.t()
    gate, up = gr.chunk(2, dim=-1)
    (torch.nn.functional.silu(gate) * up).backward(gh.float())
    assert_bf16_close(xd.grad, xr.grad, what="grad_x")
    assert_bf16_close(wd.grad, wr.grad, what="grad_w")


def test_gate_up_swiglu_in_model_matches_unfused(cuda_device):
    """The model's gate_up module on the fused kernel equals the unfused b200 path
    (GEMM + standalone SwiGLU kernel) on the same weights."""
    from hackable_lm_b200 import kernels, ops

    x, w, gh = _operands(512, 768, 2048, seed=1)
    xd, wd = x.to(cuda_device), w.to(cuda_device)
    h_fused, _ = ops.gate_up_swiglu(xd, wd)
    h_unfused = kernels.swiglu_triton(torch.nn.functional.linear(xd, wd))
    assert_bf16_close(h_fused, h_unfused.float(), what="fused vs unfused")


def test_gate_up_swiglu_rejects_cpu():
    from hackable_lm_b200 import ops

    x, w, _ = _operands(256, 128, 128)
    with pytest.raises(Exception):
        ops.gate_up_swiglu(x, w)


@pytest.mark.parametrize("M,C,H", [(256, 256, 256), (300, 768, 512), (4096, 768, 2048), (1000, 128, 256)])
def test_mlp_down_backward_fused_vs_oracle(M, C, H, cuda_device):
    """gate_up_swiglu -> swiglu_down: forward y and the gradients of x, W_gate_up and W_down,
    with the down projection's backward computing grad_h and the SwiGLU backward in one
    kernel, against fp32 autograd of the same bf16 operands."""
    from hackable_lm_b200 import _lib, ops

    _lib.clear_device_error()
    x, w, _ = _operands(M, C, H, seed=2)
    g = torch.Generator().manual_seed(3)
    wd = (torch.randn(C, H, generator=g) * 0.02).to(torch.bfloat16)
    gy = torch.randn(M, C, generator=g).to(torch.bfloat16)
    xd = x.to(cuda_device).requires_grad_(True)
    wgd = w.to(cuda_device).requires_grad_(True)
    wdd = wd.to(cuda_device).requires_grad_(True)
    h, gate_up = ops.gate_up_swiglu(xd, wgd)
    y = ops.swiglu_down(h, gate_up, wdd)
    y.backward(gy.to(cuda_device))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0

    xr = x.float().requires_grad_(True)
    wr = w.float().requires_grad_(True)
    wdr = wd.float().requires_grad_(True)
    gate, up = (xr @ wr.t()).chunk(2, dim=-1)
    yr = (torch.nn.functional.silu(gate) * up) @ wdr.t()
    yr.backward(gy.float())
    assert_bf16_close(y, yr, what="y")
    assert_bf16_close(xd.grad, xr.grad, what="grad_x")
    assert_bf16_close(wgd.grad, wr.grad, what="grad_w_gate_up")
    assert_bf16_close(wdd.grad, wdr.grad, what="grad_w_down")


def test_swiglu_down_bwd_kernel_matches_unfused(cuda_device):
    """The fused kernel's grad_gate_up equals the unfused composition (cuBLAS grad_h in bf16,
    then the standalone SwiGLU backward kernel) up to the GEMM's accumulation order."""
    from hackable_lm_b200 import _lib, ops

    M, C, H = 2048, 768, 2048
    g = torch.Generator().manual_seed(4)
    gate_up = torch.randn(M, 2 * H, generator=g).to(torch.bfloat16).to(cuda_device)
    wd = (torch.randn(C, H, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    gy = torch.randn(M, C, generator=g).to(torch.bfloat16).to(cuda_device)
    out = torch.empty_like(gate_up)
    _lib.check(_lib.load().hlm_swiglu_down_bwd(gy.data_ptr(), wd.data_ptr(), gate_up.data_ptr(),
                                                out.data_ptr(), M, C, H, 0), "hlm_swiglu_down_bwd")
    ref = ops.swiglu_backward(gate_up, gy @ wd)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert_bf16_close(out, ref.float(), what="grad_gate_up")


def test_swiglu_down_rejects_cpu():
    from hackable_lm_b200 import ops

    h = torch.zeros(4, 256, dtype=torch.bfloat16)
    with pytest.raises(Exception):
        ops.swiglu_down(h, torch.zeros(4, 512, dtype=torch.bfloat16), torch.zeros(64, 256, dtype=torch.bfloat16))
