"""Attention core: the tcgen05 forward (causal, sliding window) against an fp32
explicit-softmax reference (the reference's "torch" attention, kernels.py:785-800,
with the window mask of model.py:143-153), its log-sum-exp, and gradients through the
cuDNN backward fed with this forward's output and statistics."""
from __future__ import annotations

import math

import pytest
import torch

from parity import assert_bf16_close

pytestmark = pytest.mark.gpu


def _ref(q, k, v, window):
    """fp32 attention on [B, T, H, D] (k/v heads repeated for grouped queries)."""
    B, T, H, D = q.shape
    rep = H // k.shape[2]
    qf = q.float().transpose(1, 2)
    kf = k.float().repeat_interleave(rep, dim=2).transpose(1, 2)
    vf = v.float().repeat_interleave(rep, dim=2).transpose(1, 2)
    s = qf @ kf.transpose(-1, -2) / math.sqrt(D)
    pos = torch.arange(T, device=q.device)
    dist = pos[:, None] - pos[None, :]
    keep = (dist >= 0) & (dist < (window if window > 0 else T))
    s = s.masked_fill(~keep, float("-inf"))
    lse = torch.logsumexp(s, -1)
    return (torch.softmax(s, -1) @ vf).transpose(1, 2), lse


def _inputs(B, T, H, Hk, seed, dev):
    g = torch.Generator().manual_seed(seed)
    mk = lambda h: torch.randn(B, T, h, 128, generator=g).to(torch.bfloat16).to(dev)  # noqa: E731
    return mk(H), mk(Hk), mk(Hk)


@pytest.mark.parametrize("B,T,H,Hk,window", [(2, 256, 2, 2, 0), (1, 512, 3, 3, 128), (2, 384, 2, 2, 200),
                                             (1, 640, 4, 2, 0), (1, 1024, 1, 1, 512), (1, 128, 1, 1, 0),
                                             (1, 256, 1, 1, 1)])
def test_attention_forward_vs_reference(B, T, H, Hk, window, cuda_device):
    from hackable_lm_b200 import _lib, ops

    _lib.clear_device_error()
    q, k, v = _inputs(B, T, H, Hk, 0, cuda_device)
    out, lse = ops.attention(q, k, v, window, 1.0 / math.sqrt(128))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    ref, ref_lse = _ref(q, k, v, window)
    assert_bf16_close(out, ref, what="out")
    torch.testing.assert_close(lse, ref_lse, atol=2e-2, rtol=0, msg=lambda m: f"lse: {m}")


@pytest.mark.parametrize("slope,window", [(0.9, 0), (1.2, 0), (3.0, 0), (0.9, 300)])
def test_attention_forward_rising_scores(slope, window, cuda_device):
    """Scores that rise along the keys by `slope` (log2 units per key): every key tile
    exceeds the running reference max by far more than the in-range bound, so the
    kernel leaves its fast path (no row max) for the exact path (first half out of
    range) or moves the reference after publishing the first half (second half out
    of range), and must still match the fp32 softmax."""
    from hackable_lm_b200 import _lib, ops

    _lib.clear_device_error()
    B, T, H = 1, 512, 2
    beta = slope * math.sqrt(128) / math.log2(math.e)
    q = torch.zeros(B, T, H, 128)
    q[..., 0] = 1.0
    k = torch.zeros(B, T, H, 128)
    k[..., 0] = beta * torch.arange(T, dtype=torch.float32)[None, :, None]
    g = torch.Generator().manual_seed(5)
    v = torch.randn(B, T, H, 128, generator=g)
    q, k, v = (t.to(torch.bfloat16).to(cuda_device) for t in (q, k, v))
    out, lse = ops.attention(q, k, v, window, 1.0 / math.sqrt(128))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.isfinite(out.float()).all() and torch.isfinite(lse).all()
    ref, ref_lse = _ref(q, k, v, window)
    assert_bf16_close(out, ref, what="out")
    torch.testing.assert_close(lse, ref_lse, atol=2e-2, rtol=1e-5, msg=lambda m: f"lse: {m}")


def _sdpa_grads(q, k, v, go, window):
    """Gradients of torch SDPA (cuDNN on B200) on the same bf16 inputs."""
    T = q.shape[1]
    qs, ks, vs = (t.clone().transpose(1, 2).requires_grad_(True) for t in (q, k, v))
    mask = None
    if window > 0:
        pos = torch.arange(T, device=q.device)
        dist = pos[:, None] - pos[None, :]
        mask = (dist >= 0) & (dist < window)
    out = torch.nn.functional.scaled_dot_product_attention(qs, ks, vs, attn_mask=mask, is_causal=mask is None)
    out.backward(go.transpose(1, 2))
    return [t.grad.transpose(1, 2) for t in (qs, ks, vs)]


def _rel_l2(a, e):
    a, e = a.double(), e.double()
    return ((a - e).norm() / e.norm()).item()


@pytest.mark.parametrize("T,window", [(256, 0), (512, 160)])
def test_attention_backward_vs_reference(T, window, cuda_device):
    """Gradients against fp32 autograd: relative L2 within 1e-2 and no further than 1.5x
    (+2e-3) the error of torch SDPA's own bf16 gradients on the same inputs (the
    elementwise bf16 bar does not hold for attention gradients even for SDPA itself)."""
    from hackable_lm_b200 import ops
    from parity import record

    q, k, v = _inputs(2, T, 2, 2, 1, cuda_device)
    g = torch.Generator().manual_seed(2)
    go = torch.randn(2, T, 2, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    out, _ = ops.attention(qd, kd, vd, window, 1.0 / math.sqrt(128))
    out.backward(go)
    qr, kr, vr = (t.float().requires_grad_(True) for t in (q, k, v))
    ref, _ = _ref(qr, kr, vr, window)
    ref.backward(go.float())
    sdpa = _sdpa_grads(q, k, v, go, window)
    for name, got, exp, other in zip("qkv", (qd.grad, kd.grad, vd.grad), (qr.grad, kr.grad, vr.grad), sdpa):
        e_ours, e_sdpa = _rel_l2(got, exp), _rel_l2(other, exp)
        record(f"attention grad_{name}", rel_l2=e_ours, sdpa_rel_l2=e_sdpa)
        assert e_ours <= 1e-2 and e_ours <= 1.5 * e_sdpa + 2e-3, (name, e_ours, e_sdpa)


def test_attention_d12_shape_vs_sdpa(cuda_device):
    """d12 shape [16, 2048, 6, 128], full causal: output, lse and gradients against
    torch SDPA (cuDNN) on the same inputs."""
    from hackable_lm_b200 import _lib, ops

    _lib.clear_device_error()
    q, k, v = _inputs(16, 2048, 6, 6, 3, cuda_device)
    g = torch.Generator().manual_seed(4)
    go = torch.randn(16, 2048, 6, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    out, lse = ops.attention(qd, kd, vd, 0, 1.0 / math.sqrt(128))
    out.backward(go)
    qs, ks, vs = (t.clone().transpose(1, 2).requires_grad_(True) for t in (q, k, v))
    ref = torch.nn.functional.scaled_dot_product_attention(qs, ks, vs, is_causal=True)
    ref.backward(go.transpose(1, 2))
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert_bf16_close(out, ref.transpose(1, 2).float(), what="out")
    for name, a, e in zip("qkv", (qd.grad, kd.grad, vd.grad), (qs.grad, ks.grad, vs.grad)):
        # both bf16; the backward kernel is the same, fed with either forward's statistics
        assert _rel_l2(a, e.transpose(1, 2)) <= 1e-2, (name, _rel_l2(a, e.transpose(1, 2)))


@pytest.mark.parametrize("backend,bwd", [("flash_attn_2", "auto"), ("sdpa", "auto"), ("sdpa", "library")])
def test_sliding_window_takes_the_b200_path(backend, bwd, cuda_device):
    """The reference entry point with a sliding window (its default pattern) runs the
    tcgen05 forward under every backend name but "torch", and its gradients (the tcgen05
    backward by default; flash_attn's windowed backward, or cuDNN with the window as a
    bias, in "library" mode) match the fp32 reference within the bar SDPA's own bf16
    gradients set."""
    from hackable_lm_b200 import _lib, kernels, ops

    _lib.clear_device_error()
    B, T, H, W = 2, 512, 2, 160
    q, k, v = _inputs(B, T, H, H, 6, cuda_device)
    g = torch.Generator().manual_seed(7)
    go = torch.randn(B, T, H, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    qd, kd, vd = (t.clone().requires_grad_(True) for t in (q, k, v))
    flash = backend.startswith("flash")
    args = (qd, kd, vd) if flash else tuple(t.transpose(1, 2) for t in (qd, kd, vd))
    with _lib.KernelTimer("attn_fwd", 4) as timer:
        out = kernels.scaled_dot_product_attention(*args, 0.0, is_causal=True, window_size=W, backend=backend)
    out = out if flash else out.transpose(1, 2)
    old = ops.ATTENTION_BWD["mode"]
    ops.ATTENTION_BWD["mode"] = bwd
    try:
        with _lib.KernelTimer("attn_bwd", 8) as btimer:
            out.backward(go)
    finally:
        ops.ATTENTION_BWD["mode"] = old
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert timer.launches == 1
    assert btimer.launches == (3 if bwd == "auto" else 0)
    ref, _ = _ref(q, k, v, W)
    assert_bf16_close(out, ref, what="out")
    qr, kr, vr = (t.float().clone().requires_grad_(True) for t in (q, k, v))
    ref_out, _ = _ref(qr, kr, vr, W)
    ref_out.backward(go.float())
    for name, a, e, s in zip("qkv", (qd.grad, kd.grad, vd.grad), (qr.grad, kr.grad, vr.grad),
                             _sdpa_grads(q, k, v, go, W)):
        sdpa_err = _rel_l2(s, e)
        assert _rel_l2(a, e) <= 2 * sdpa_err + 1e-3, (name, _rel_l2(a, e), sdpa_err)


@pytest.mark.parametrize("B,T,H,window", [(2, 256, 2, 0), (2, 512, 2, 160), (1, 384, 2, 200), (1, 1024, 1, 512),
                                          (1, 128, 1, 0), (2, 512, 2, 1)])
def test_attention_native_backward_vs_reference(B, T, H, window, cuda_device):
    """hlm_attention_bwd (the tcgen05 backward) against fp32 gradients, within twice
    the error SDPA's own bf16 gradients have on the same inputs."""
    from hackable_lm_b200 import _lib, ops

    _lib.clear_device_error()
    q, k, v = _inputs(B, T, H, H, 8, cuda_device)
    g = torch.Generator().manual_seed(9)
    go = torch.randn(B, T, H, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    scale = 1.0 / math.sqrt(128)
    out, lse = ops.attention(q, k, v, window, scale)
    old = ops.ATTENTION_BWD["mode"]
    ops.ATTENTION_BWD["mode"] = "native"
    try:
        with _lib.KernelTimer("attn_bwd", 8) as timer:
            dq, dk, dv = ops.attention_backward(go, q, k, v, out, lse, window, scale)
    finally:
        ops.ATTENTION_BWD["mode"] = old
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert timer.launches == 3
    qr, kr, vr = (t.float().clone().requires_grad_(True) for t in (q, k, v))
    ref_out, _ = _ref(qr, kr, vr, window)
    ref_out.backward(go.float())
    for name, a, e, s in zip("qkv", (dq, dk, dv), (qr.grad, kr.grad, vr.grad), _sdpa_grads(q, k, v, go, window)):
        sdpa_err = _rel_l2(s, e)
        assert _rel_l2(a, e) <= 2 * sdpa_err + 1e-3, (name, _rel_l2(a, e), sdpa_err)


def test_attention_native_backward_argument_checks(cuda_device):
    """hlm_attention_bwd refuses what it does not handle before any launch: grouped
    heads, head_dim other than 128, T not a multiple of 128 (HLM_ERR_UNSUPPORTED), a
    workspace below hlm_attention_bwd_workspace_bytes or a null pointer
    (HLM_ERR_INVALID_ARG); B == 0 is a no-op."""
    from hackable_lm_b200 import _lib

    lib = _lib.load()
    B, T, H = 1, 256, 2
    t = torch.zeros(B, T, H, 128, dtype=torch.bfloat16, device=cuda_device)
    lse = torch.zeros(B, H, T, dtype=torch.float32, device=cuda_device)
    need = int(lib.hlm_attention_bwd_workspace_bytes(B, T, H, 128))
    assert need == B * T * H * 128 * 4 + B * H * T * 8 + 256
    ws = torch.empty(need, dtype=torch.uint8, device=cuda_device)
    outs = [torch.empty_like(t) for _ in range(3)]
    stream = torch.cuda.current_stream(cuda_device).cuda_stream

    def call(nbytes=need, B_=B, T_=T, Hk=H, D=128, ws_ptr=ws.data_ptr()):
        return lib.hlm_attention_bwd(t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(),
                                     lse.data_ptr(), *(o.data_ptr() for o in outs), ws_ptr, nbytes, B_, T_, H, Hk, D,
                                     0, 0.088, stream)

    assert call(Hk=1) == -2
    assert call(D=64) == -2
    assert call(T_=200) == -2
    assert call(nbytes=need - 16) == -1
    assert call(ws_ptr=0) == -1
    assert call(B_=0) == 0
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
