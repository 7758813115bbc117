"""Fused LM head + cross-entropy: parity with the CPU oracle (small shapes and the
golden vectors), and at the full BASELINE config 4 size against a chunked
PyTorch fp32 computation plus a size-independent identity."""
from __future__ import annotations

import pytest
import torch

import oracle
from parity import assert_bf16_close, assert_loss_close

pytestmark = pytest.mark.gpu


def _run(hidden, weight, targets, ignore_index, device):
    from hackable_lm_b200 import kernels

    h = hidden.to(device).requires_grad_(True)
    w = weight.to(device).requires_grad_(True)
    loss = kernels.fused_linear_cross_entropy_with_weight(h, w, None, targets.to(device), "triton",
                                                          chunk_size=4096, ignore_index=ignore_index)
    loss.backward()
    return loss.detach(), h.grad, w.grad


@pytest.mark.parametrize("n,C,V,ignore_frac", [(300, 64, 520, 0.0), (1024, 256, 4096, 0.02),
                                               (130, 128, 1000, 0.1), (2048, 768, 8192, 0.02)])
def test_lm_head_vs_oracle(n, C, V, ignore_frac, cuda_device):
    from hackable_lm_b200 import _lib

    _lib.clear_device_error()
    g = torch.Generator().manual_seed(0)
    hidden = torch.randn(n, C, generator=g).to(torch.bfloat16)
    weight = (torch.randn(V, C, generator=g) * 0.02).to(torch.bfloat16)
    targets = torch.randint(0, V, (n,), generator=g)
    n_ign = int(round(ignore_frac * n))
    if n_ign:
        targets[torch.randperm(n, generator=g)[:n_ign]] = -1
    loss, gx, gw = _run(hidden, weight, targets, -1, cuda_device)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    o_loss, o_gx, o_gw = oracle.lm_head_ce(hidden, weight, targets, -1, 0)
    assert_loss_close(loss, o_loss)
    assert_bf16_close(gx, o_gx, what="grad_hidden")
    assert_bf16_close(gw, o_gw, what="grad_weight")
    if n_ign:
        assert torch.count_nonzero(gx[targets.to(gx.device) == -1]) == 0


def test_lm_head_golden_ignore(golden, cuda_device):
    gd = golden("lm_head")["dense_ignore"]
    # C must be a multiple of 64 and V of 8: the golden case is 64 x 96
    loss, gx, gw = _run(gd["hidden"].to(torch.bfloat16), gd["weight"].to(torch.bfloat16), gd["targets"],
                        gd["ignore_index"], cuda_device)
    # the fixture's hidden and weight hold bf16 values, so both sides start from the same numbers
    assert_loss_close(loss, gd["loss"])
    assert_bf16_close(gx, gd["grad_hidden"], what="grad_hidden")
    assert_bf16_close(gw, gd["grad_weight"], what="grad_weight")


def test_lm_head_grad_output_scaling(cuda_device):
    from hackable_lm_b200 import kernels

    g = torch.Generator().manual_seed(3)
    hidden = torch.randn(256, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    weight = (torch.randn(512, 128, generator=g) * 0.02).to(torch.bfloat16).to(cuda_device)
    targets = torch.randint(0, 512, (256,), generator=g).to(cuda_device)
    h1 = hidden.clone().requires_grad_(True)
    l1 = kernels.fused_linear_cross_entropy_with_weight(h1, weight, None, targets, "b200")
    (l1 * 3.0).backward()
    h2 = hidden.clone().requires_grad_(True)
    l2 = kernels.fused_linear_cross_entropy_with_weight(h2, weight, None, targets, "b200")
    l2.backward()
    torch.testing.assert_close(h1.grad.float(), 3.0 * h2.grad.float(), atol=1e-2, rtol=1e-2)


def test_lm_head_c4_full_size(cuda_device):
    """hidden [32768,768], W [32768,768], 2% ignore_index=-1."""
    from hackable_lm_b200 import _lib

    _lib.clear_device_error()
    M, C, V = 32768, 768, 32768
    g = torch.Generator().manual_seed(0)
    hidden = torch.randn(M, C, generator=g).to(torch.bfloat16)
    weight = (torch.randn(V, C, generator=g) * 0.02).to(torch.bfloat16)
    targets = torch.randint(0, V, (M,), generator=g)
    targets[torch.randperm(M, generator=g)[: int(0.02 * M)]] = -1
    loss, gx, gw = _run(hidden, weight, targets, -1, cuda_device)
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    # fp32 reference on the GPU, chunked over tokens
    h = hidden.to(cuda_device).float()
    w = weight.to(cuda_device).float()
    t = targets.to(cuda_device)
    valid = t != -1
    nv = int(valid.sum())
    loss_sum = torch.zeros((), device=cuda_device, dtype=torch.float64)
    ref_gx = torch.empty_like(h)
    ref_gw = torch.zeros_like(w)
    for s in range(0, M, 4096):
        lg = h[s:s + 4096] @ w.t()
        tc = t[s:s + 4096]
        loss_sum += torch.nn.functional.cross_entropy(lg, tc, ignore_index=-1, reduction="sum").double()
        p = torch.softmax(lg, dim=-1)
        vm = valid[s:s + 4096]
        rows = torch.nonzero(vm).squeeze(-1)
        p[rows, tc[rows]] -= 1.0
        p[~vm] = 0.0
        p /= nv
        ref_gx[s:s + 4096] = p @ w
        ref_gw += p.t() @ h[s:s + 4096]
    assert_loss_close(loss, loss_sum / nv)
    assert_bf16_close(gx, ref_gx, what="grad_hidden")
    assert_bf16_close(gw, ref_gw, what="grad_weight")
    # identity independent of size: <dX, H> = <dW, W> = sum(dlogits * logits)
    lhs = (gx.double() * hidden.to(cuda_device).double()).sum()
    rhs = (gw.double() * weight.to(cuda_device).double()).sum()
    assert abs(lhs - rhs).item() <= 2e-2 * max(abs(lhs).item(), abs(rhs).item(), 1e-6)
