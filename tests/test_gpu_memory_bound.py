"""GPU parity of the memory-bound kernels (SwiGLU, residual-add + RMSNorm,
QK-norm + RoPE) against the CPU oracle and the reference golden vectors."""
from __future__ import annotations

import pytest
import torch

import oracle
from parity import assert_bf16_close, assert_fp32_close

pytestmark = pytest.mark.gpu


def _dev_err_zero():
    from hackable_lm_b200 import _lib

    torch.cuda.synchronize()
    assert _lib.device_error() == 0


def seeded(*shape, seed=0, std=1.0, mean=0.0):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g) * std + mean


# ----------------------------------------------------------------- SwiGLU
def test_swiglu_golden_fp32(golden, cuda_device):
    from hackable_lm_b200 import kernels

    for case in golden("swiglu")["cases"]:
        x = case["gate_up"].to(cuda_device).requires_grad_(True)
        out = kernels.swiglu_triton(x)
        out.backward(case["grad_out"].to(cuda_device))
        assert_fp32_close(out, case["out"], what="swiglu out")
        assert_fp32_close(x.grad, case["grad_gate_up"], what="swiglu grad")


@pytest.mark.parametrize("shape", [(128, 4096), (3, 7, 2 * 1000), (16384, 4096)])
def test_swiglu_bf16_vs_oracle(shape, cuda_device):
    from hackable_lm_b200 import kernels

    gate_up = seeded(*shape).to(torch.bfloat16)
    grad = seeded(*shape[:-1], shape[-1] // 2, seed=1).to(torch.bfloat16)
    x = gate_up.to(cuda_device).requires_grad_(True)
    out = kernels.swiglu_triton(x)
    out.backward(grad.to(cuda_device))
    assert out.dtype == torch.bfloat16 and x.grad.dtype == torch.bfloat16
    assert_bf16_close(out, oracle.swiglu(gate_up), what="swiglu out")
    assert_bf16_close(x.grad, oracle.swiglu_backward(gate_up, grad), what="swiglu grad")
    _dev_err_zero()


def test_swiglu_rejects_odd_width(cuda_device):
    from hackable_lm_b200 import kernels

    with pytest.raises(RuntimeError):
        kernels.swiglu_triton(torch.zeros(4, 7, device=cuda_device))


# ----------------------------------------------------------------- RMSNorm
def test_rmsnorm_c1_fp32_golden(golden, cuda_device):
    """[4,256,384] fp32 with weight, forward + backward."""
    from hackable_lm_b200 import ops

    gd = golden("rmsnorm_c1")
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4, 256, 384, generator=g)
    residual = torch.randn(4, 256, 384, generator=g)
    weight = 1.0 + torch.randn(384, generator=g) * 0.02
    grad = torch.randn(4, 256, 384, generator=g)
    xr = x.to(cuda_device).requires_grad_(True)
    rr = residual.to(cuda_device).requires_grad_(True)
    wr = weight.to(cuda_device).requires_grad_(True)
    out, norm = ops.residual_rms_norm(rr, xr, wr, 1e-6)
    norm.backward(grad.to(cuda_device))
    rows = gd["rows"]
    flat = lambda t: t.detach().reshape(1024, 384)[rows.to(t.device)]  # noqa: E731
    assert_fp32_close(flat(out), gd["out"], what="out")
    assert_fp32_close(flat(norm), gd["norm"], what="norm")
    assert_fp32_close(flat(xr.grad), gd["grad_x"], what="grad_x")
    assert_fp32_close(flat(rr.grad), gd["grad_residual"], what="grad_residual")
    torch.testing.assert_close(wr.grad.cpu().double(), gd["grad_weight"].double(), atol=5e-4, rtol=1e-5)
    _dev_err_zero()


@pytest.mark.parametrize("rows,cols", [(32768, 768), (1000, 384), (37, 100), (8, 2048)])
def test_residual_rms_norm_bf16_vs_oracle(rows, cols, cuda_device):
    from hackable_lm_b200 import kernels

    residual = seeded(rows, cols).to(torch.bfloat16)
    branch = seeded(rows, cols, seed=1).to(torch.bfloat16)
    g_out = seeded(rows, cols, seed=2).to(torch.bfloat16)
    g_norm = seeded(rows, cols, seed=3).to(torch.bfloat16)
    r = residual.to(cuda_device).requires_grad_(True)
    b = branch.to(cuda_device).requires_grad_(True)
    out, norm = kernels.residual_rms_norm(r, b, 1e-6)
    torch.autograd.backward((out, norm), (g_out.to(cuda_device), g_norm.to(cuda_device)))
    o_out, o_norm = oracle.residual_rms_norm(residual, branch, 1e-6)
    assert torch.equal(out.cpu(), o_out.to(torch.bfloat16)), "residual add must be exact in bf16"
    assert_bf16_close(norm, o_norm, what="norm")
    dx, _ = oracle.residual_rms_norm_backward(o_out, g_out, g_norm, 1e-6)
    assert_bf16_close(r.grad, dx, what="grad residual")
    assert_bf16_close(b.grad, dx, what="grad branch")
    _dev_err_zero()


def test_rms_norm_plain_weightless(cuda_device):
    from hackable_lm_b200 import kernels

    x = seeded(64, 768).to(torch.bfloat16)
    y = kernels.rms_norm(x.to(cuda_device), None, 1e-6)
    assert_bf16_close(y, oracle.rms_norm(x, None, 1e-6), what="rms_norm")


# ----------------------------------------------------------------- QK-norm + RoPE
def test_qk_norm_rope_golden(golden, cuda_device):
    from hackable_lm_b200 import kernels

    for case in golden("qk_norm_rope")["cases"]:
        q = case["q"].to(cuda_device).requires_grad_(True)
        k = case["k"].to(cuda_device).requires_grad_(True)
        qo, ko = kernels.qk_norm_rope_triton(q, k, case["cos"].to(cuda_device), case["sin"].to(cuda_device),
                                             case["eps"])
        ((qo * case["grad_q_out"].to(cuda_device)).sum() + (ko * case["grad_k_out"].to(cuda_device)).sum()).backward()
        assert_fp32_close(qo, case["q_out"], tol=2e-5, what="q_out")
        assert_fp32_close(ko, case["k_out"], tol=2e-5, what="k_out")
        assert_fp32_close(q.grad, case["grad_q"], tol=5e-5, what="grad_q")
        assert_fp32_close(k.grad, case["grad_k"], tol=5e-5, what="grad_k")
    _dev_err_zero()


@pytest.mark.parametrize("fraction", [0.25, 1.0])
def test_qk_norm_rope_c2_strided_bf16(fraction, cuda_device):
    """BASELINE config 2 RoPE: q,k [8,2048,6,128] bf16, base 1e4, read as strided
    views of a packed qkv tensor (row stride 2304) as in QKVProjection._project."""
    from hackable_lm_b200 import kernels

    B, T, H, D = 8, 2048, 6, 128
    qkv = seeded(B, T, 3 * H * D).to(torch.bfloat16)
    cos, sin = oracle.rope_tables(D, T, 10_000.0, fraction, dtype=torch.bfloat16)
    dq = seeded(B, T, H, D, seed=1).to(torch.bfloat16)
    dk = seeded(B, T, H, D, seed=2).to(torch.bfloat16)
    qkv_d = qkv.to(cuda_device).requires_grad_(True)
    q, k, _ = qkv_d.split((H * D, H * D, H * D), dim=-1)
    q = q.view(B, T, H, D)
    k = k.view(B, T, H, D)
    qo, ko = kernels.qk_norm_rope_triton(q, k, cos.transpose(1, 2).to(cuda_device),
                                         sin.transpose(1, 2).to(cuda_device), 1e-6)
    assert qo.is_contiguous() and ko.is_contiguous()
    ((qo.float() * dq.to(cuda_device).float()).sum() + (ko.float() * dk.to(cuda_device).float()).sum()).backward()
    qc, kc, _ = qkv.split((H * D, H * D, H * D), dim=-1)
    qc = qc.reshape(B, T, H, D)
    kc = kc.reshape(B, T, H, D)
    oq, ok_ = oracle.qk_norm_rope(qc, kc, cos, sin, 1e-6)
    assert_bf16_close(qo, oq, what="q_out")
    assert_bf16_close(ko, ok_, what="k_out")
    gq, gk = oracle.qk_norm_rope_backward(qc, kc, dq, dk, cos, sin, 1e-6)
    gqkv = qkv_d.grad.cpu()
    assert_bf16_close(gqkv[..., : H * D].reshape(B, T, H, D), gq, what="grad q")
    assert_bf16_close(gqkv[..., H * D: 2 * H * D].reshape(B, T, H, D), gk, what="grad k")
    assert torch.count_nonzero(gqkv[..., 2 * H * D:]) == 0
    _dev_err_zero()


@pytest.mark.parametrize("B,T,Hq,Hk,D,fraction,cs_dtype", [
    (3, 1000, 4, 2, 64, 0.25, torch.bfloat16),    # 4 lanes per head vector, rotary_dim 16
    (2, 1500, 2, 1, 256, 0.5, torch.float32),     # 16 lanes per head vector, fp32 cos/sin
    (4, 700, 3, 3, 128, 0.125, torch.bfloat16),   # rotary_dim 16: one rotated lane per head
    (5, 900, 6, 6, 128, 0.0, torch.bfloat16),     # no rotation: norm only
])
def test_qk_norm_rope_vec_layouts_bf16(B, T, Hq, Hk, D, fraction, cs_dtype, cuda_device):
    """Lane layouts of the vector kernel other than the C2 shape (head dims 64 and
    256, GQA head counts, fp32 tables, rotary_dim 16 and 0), forward and backward,
    with more tokens than resident warps so that every warp walks several tokens."""
    from hackable_lm_b200 import kernels

    q = seeded(B, T, Hq, D).to(torch.bfloat16)
    k = seeded(B, T, Hk, D, seed=3).to(torch.bfloat16)
    dq = seeded(B, T, Hq, D, seed=1).to(torch.bfloat16)
    dk = seeded(B, T, Hk, D, seed=2).to(torch.bfloat16)
    cos, sin = oracle.rope_tables(D, T, 10_000.0, fraction, dtype=cs_dtype)
    qd = q.to(cuda_device).requires_grad_(True)
    kd = k.to(cuda_device).requires_grad_(True)
    qo, ko = kernels.qk_norm_rope_triton(qd, kd, cos.transpose(1, 2).to(cuda_device),
                                         sin.transpose(1, 2).to(cuda_device), 1e-6)
    torch.autograd.backward((qo, ko), (dq.to(cuda_device), dk.to(cuda_device)))
    oq, ok_ = oracle.qk_norm_rope(q, k, cos, sin, 1e-6)
    assert_bf16_close(qo, oq, what="q_out")
    assert_bf16_close(ko, ok_, what="k_out")
    gq, gk = oracle.qk_norm_rope_backward(q, k, dq, dk, cos, sin, 1e-6)
    assert_bf16_close(qd.grad, gq, what="grad q")
    assert_bf16_close(kd.grad, gk, what="grad k")
    _dev_err_zero()
