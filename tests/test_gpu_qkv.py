"""Fused QKV projection + QK-norm + RoPE: forward and backward parity."""
from __future__ import annotations

import pytest
import torch

import oracle
from parity import assert_bf16_close

pytestmark = pytest.mark.gpu


def _inputs(B, T, C, H, Hk, fraction, theta, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, C, generator=g).to(torch.bfloat16)
    w = (torch.randn((H + 2 * Hk) * 128, C, generator=g) * 0.02).to(torch.bfloat16)
    cos, sin = oracle.rope_tables(128, T, theta, fraction, dtype=torch.bfloat16)
    dq = torch.randn(B, T, H, 128, generator=g).to(torch.bfloat16)
    dk = torch.randn(B, T, Hk, 128, generator=g).to(torch.bfloat16)
    dv = torch.randn(B, T, Hk, 128, generator=g).to(torch.bfloat16)
    return x, w, cos, sin, dq, dk, dv


def _run(x, w, cos, sin, dq, dk, dv, H, Hk, dev):
    from hackable_lm_b200 import kernels

    xr = x.to(dev).requires_grad_(True)
    wr = w.to(dev).requires_grad_(True)
    q, k, v = kernels.qkv_projection_rope(xr, wr, cos.to(dev), sin.to(dev), H, Hk, 1e-6)
    torch.autograd.backward((q, k, v), (dq.to(dev), dk.to(dev), dv.to(dev)))
    return q, k, v, xr.grad, wr.grad


@pytest.mark.parametrize("B,T,C,H,Hk,fraction", [(2, 64, 256, 2, 2, 0.25), (1, 200, 768, 6, 6, 1.0),
                                                 (2, 128, 512, 4, 2, 0.25), (2, 96, 768, 6, 6, 0.5)])
def test_qkv_vs_oracle(B, T, C, H, Hk, fraction, cuda_device):
    from hackable_lm_b200 import _lib

    _lib.clear_device_error()
    x, w, cos, sin, dq, dk, dv = _inputs(B, T, C, H, Hk, fraction, 10_000.0)
    q, k, v, gx, gw = _run(x, w, cos, sin, dq, dk, dv, H, Hk, cuda_device)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    oq, ok_, ov = oracle.qkv_rope(x, w, cos, sin, H, Hk, 1e-6)
    assert_bf16_close(q, oq, what="q")
    assert_bf16_close(k, ok_, what="k")
    assert_bf16_close(v, ov, what="v")
    ogx, ogw = oracle.qkv_rope_backward(x, w, cos, sin, dq, dk, dv, H, Hk, 1e-6)
    assert_bf16_close(gx, ogx, what="grad_x")
    assert_bf16_close(gw, ogw, what="grad_w")


def test_qkv_golden(golden, cuda_device):
    gd = golden("qkv")
    x = gd["x"].to(torch.bfloat16)
    w = gd["w_qkv"].to(torch.bfloat16)
    # the fixture's x, w and upstream grads hold bf16 values (exact in bf16); cos/sin stay
    # fp32 as the reference module computed them
    q, k, v, gx, gw = _run(x, w, gd["cos"], gd["sin"],
                           gd["grad_q_out"].to(torch.bfloat16), gd["grad_k_out"].to(torch.bfloat16),
                           gd["grad_v_out"].to(torch.bfloat16), gd["n_head"], gd["n_kv_head"], cuda_device)
    assert_bf16_close(q, gd["q"], what="q")
    assert_bf16_close(k, gd["k"], what="k")
    assert_bf16_close(v, gd["v"], what="v")
    assert_bf16_close(gx, gd["grad_x"], what="grad_x")
    assert_bf16_close(gw, gd["grad_w"], what="grad_w")


def test_qkv_c3_full_size(cuda_device):
    """X [16384,768] (8 x 2048), W [2304,768], 6+6+6 heads, base 1e4."""
    B, T, C, H = 8, 2048, 768, 6
    x, w, cos, sin, dq, dk, dv = _inputs(B, T, C, H, H, 0.25, 10_000.0)
    q, k, v, gx, gw = _run(x, w, cos, sin, dq, dk, dv, H, H, cuda_device)
    # torch fp32 reference on the GPU (same formulas as the oracle)
    dev = cuda_device
    xr = x.to(dev).float().requires_grad_(True)
    wr = w.to(dev).float().requires_grad_(True)
    qkv = xr @ wr.t()
    rq, rk, rv = qkv.split((H * 128, H * 128, H * 128), dim=-1)
    rq = rq.reshape(B, T, H, 128)
    rk = rk.reshape(B, T, H, 128)
    rv = rv.reshape(B, T, H, 128)
    c = cos.to(dev).float().transpose(1, 2)
    s = sin.to(dev).float().transpose(1, 2)
    rq = oracle.apply_partial_rope(rq * torch.rsqrt(rq.pow(2).mean(-1, keepdim=True) + 1e-6), c, s)
    rk = oracle.apply_partial_rope(rk * torch.rsqrt(rk.pow(2).mean(-1, keepdim=True) + 1e-6), c, s)
    torch.autograd.backward((rq, rk, rv), (dq.to(dev).float(), dk.to(dev).float(), dv.to(dev).float()))
    assert_bf16_close(q, rq, what="q")
    assert_bf16_close(k, rk, what="k")
    assert_bf16_close(v, rv, what="v")
    assert_bf16_close(gx, xr.grad, what="grad_x")
    assert_bf16_close(gw, wr.grad, what="grad_w")
