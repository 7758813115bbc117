"""Output / down projection with the residual add and RMSNorm in the GEMM epilogue
(thread-block clusters exchanging row sums), against the CPU oracle and the unfused
composition, forward and backward."""
from __future__ import annotations

import pytest
import torch

import oracle
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu


def _operands(M, K, N, seed=0):
    g = torch.Generator().manual_seed(seed)
    y = torch.randn(M, K, generator=g).to(torch.bfloat16)
    w = (torch.randn(N, K, generator=g) * 0.02).to(torch.bfloat16)
    r = torch.randn(M, N, generator=g).to(torch.bfloat16)
    go = torch.randn(M, N, generator=g).to(torch.bfloat16)
    gn = torch.randn(M, N, generator=g).to(torch.bfloat16)
    return y, w, r, go, gn


def _expected(y, w, r, eps=1e-6):
    """The reference's chain: bf16 F.linear output, bf16 residual add, RMSNorm of the bf16 sum."""
    branch = (y.float() @ w.float().t()).to(torch.bfloat16)
    out = (r.float() + branch.float()).to(torch.bfloat16)
    return out, oracle.rms_norm(out.float(), None, eps)


# N = 768 (d12: 3 CTAs x 256), 256 (one CTA), 512 (2 x 256), 1024 (4 x 256), 384 (3 x 128), 128
@pytest.mark.parametrize("M,K,N", [(300, 768, 768), (1024, 2048, 768), (200, 256, 256), (130, 512, 512),
                                   (257, 192, 1024), (96, 640, 384), (64, 128, 128), (4096, 768, 768)])
def test_proj_residual_norm_vs_oracle(M, K, N, cuda_device):
    from hackable_lm_b200 import _lib, ops

    _lib.clear_device_error()
    y, w, r, _, _ = _operands(M, K, N)
    out, norm = ops.proj_residual_norm(y.to(cuda_device), w.to(cuda_device), r.to(cuda_device), 1e-6)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    e_out, e_norm = _expected(y, w, r)
    assert_bf16_close(out, e_out.float(), what="out")
    assert_bf16_close(norm, e_norm, what="norm")


def test_proj_residual_norm_backward(cuda_device):
    from hackable_lm_b200 import ops

    M, K, N = 512, 768, 768
    y, w, r, go, gn = _operands(M, K, N, seed=1)
    dev = cuda_device
    yd, wd, rd = (t.to(dev).requires_grad_(True) for t in (y, w, r))
    out, norm = ops.proj_residual_norm(yd, wd, rd, 1e-6)
    torch.autograd.backward((out, norm), (go.to(dev), gn.to(dev)))
    yr, wr, rr = (t.float().requires_grad_(True) for t in (y, w, r))
    o = rr + yr @ wr.t()
    n = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + 1e-6)
    torch.autograd.backward((o, n), (go.float(), gn.float()))
    assert_bf16_close(yd.grad, yr.grad, what="grad_y")
    assert_bf16_close(wd.grad, wr.grad, what="grad_w")
    assert_bf16_close(rd.grad, rr.grad, what="grad_residual")


def test_swiglu_down_residual_norm_matches_unfused(cuda_device):
    """The MLP's fused down projection (residual + RMSNorm epilogue, SwiGLU-backward
    grad) equals swiglu_down followed by the residual_rms_norm kernel, values and grads."""
    from hackable_lm_b200 import kernels, ops

    g = torch.Generator().manual_seed(2)
    M, C, H = 1024, 768, 2048
    x = torch.randn(M, C, generator=g).to(torch.bfloat16).to(cuda_device)
    w_gu = (torch.randn(2 * H, C, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    w_dn = (torch.randn(C, H, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    res = torch.randn(M, C, generator=g).to(torch.bfloat16).to(cuda_device)
    go = torch.randn(M, C, generator=g).to(torch.bfloat16).to(cuda_device)
    gn = torch.randn(M, C, generator=g).to(torch.bfloat16).to(cuda_device)
    outs = []
    for fused in (True, False):
        xs, wg, wd, rs = (t.clone().requires_grad_(True) for t in (x, w_gu, w_dn, res))
        h, gate_up = ops.gate_up_swiglu(xs, wg)
        if fused:
            out, norm = ops.swiglu_down_residual_norm(h, gate_up, wd, rs, 1e-6)
        else:
            out, norm = kernels.residual_rms_norm(rs, ops.swiglu_down(h, gate_up, wd), 1e-6)
        torch.autograd.backward((out, norm), (go, gn))
        outs.append((out, norm, xs.grad, wg.grad, wd.grad, rs.grad))
    names = ("out", "norm", "grad_x", "grad_w_gate_up", "grad_w_down", "grad_residual")
    for n, a, b in zip(names, outs[0], outs[1]):
        assert_bf16_close(a, b.float(), what=n)


@pytest.mark.parametrize("K", [768, 2048])
def test_proj_residual_norm_d12_shape(K, cuda_device):
    """d12 shapes (32768 tokens; o_proj K = 768, down K = 2048) against a torch fp32
    computation of the same chain on the GPU."""
    from hackable_lm_b200 import _lib, ops

    _lib.clear_device_error()
    y, w, r, _, _ = _operands(32768, K, 768, seed=3)
    dev = cuda_device
    out, norm = ops.proj_residual_norm(y.to(dev), w.to(dev), r.to(dev), 1e-6)
    branch = (y.to(dev).float() @ w.to(dev).float().t()).to(torch.bfloat16)
    e_out = (r.to(dev).float() + branch.float()).to(torch.bfloat16).float()
    e_norm = e_out * torch.rsqrt(e_out.pow(2).mean(-1, keepdim=True) + 1e-6)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert_bf16_close(out, e_out, what="out")
    assert_bf16_close(norm, e_norm, what="norm")


def test_proj_residual_norm_rejects_unsupported(cuda_device):
    from hackable_lm_b200 import _lib, ops

    y = torch.zeros(64, 128, dtype=torch.bfloat16, device=cuda_device)
    w = torch.zeros(640, 128, dtype=torch.bfloat16, device=cuda_device)  # N = 5 x 128
    assert not ops.proj_norm_supported(y, w)
    out = torch.empty(64, 640, dtype=torch.bfloat16, device=cuda_device)
    rc = _lib.load().hlm_proj_residual_rms_norm_fwd(y.data_ptr(), w.data_ptr(), out.data_ptr(), out.data_ptr(),
                                                    out.data_ptr(), 64, 128, 640, 1e-6,
                                                    torch.cuda.current_stream().cuda_stream)
    assert rc == -2  # HLM_ERR_UNSUPPORTED
