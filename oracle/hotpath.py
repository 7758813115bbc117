"""CPU restatement of the reference hot path (test infrastructure only).

Conventions: inputs may be any floating dtype; every function upcasts to
``compute`` (float32 by default, float64 for tight checks) and returns results
in that dtype, so the GPU kernels' bf16 outputs are compared against exact
math on the same (rounded) inputs.  Gradients are either the reference's
closed forms or autograd through the reference's forward expression, as noted.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def _c(t: torch.Tensor | None, compute: torch.dtype) -> torch.Tensor | None:
    # .to() keeps the autograd graph, so qkv_rope_backward can differentiate
    # through the forward expression.
    return None if t is None else t.to("cpu", compute)


# ---------------------------------------------------------------------------
# RMSNorm and residual add  (model.py:14-16, 73-75; kernels.py:245-247)
# ---------------------------------------------------------------------------
def rms_norm(x, weight=None, eps=1e-6, compute=torch.float32):
    """y = x * rsqrt(mean(x^2, -1) + eps) [* weight]   (model.py:14-16)."""
    x = _c(x, compute)
    y = x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
    return y if weight is None else y * _c(weight, compute)


def residual_rms_norm(residual, branch, eps=1e-6, weight=None, out_dtype=None, compute=torch.float32):
    """out = residual + branch; norm = rms_norm(out)   (model.py:73-75).

    ``out`` is rounded to ``out_dtype`` (the activation dtype) before the norm,
    because the reference stores ``out`` in that dtype and normalises it.
    """
    out_dtype = out_dtype or branch.dtype
    out = (_c(residual, compute) + _c(branch, compute)).to(out_dtype).to(compute)
    return out, rms_norm(out, weight, eps, compute)


def residual_rms_norm_backward(out, grad_out, grad_norm, eps=1e-6, weight=None, compute=torch.float32):
    """Closed-form backward of norm = x*r*w with r = rsqrt(mean(x^2)+eps).

    dx = grad_out + r*(g*w) - x*r^3*mean((g*w)*x);  dweight = sum_rows g*x*r.
    Same expression as _norm_backward_no_weight (kernels.py:703-708), extended
    by the weight and the residual-stream gradient.
    """
    x = _c(out, compute)
    g = _c(grad_norm, compute)
    w = None if weight is None else _c(weight, compute)
    gw = g if w is None else g * w
    r = torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
    dot = (gw * x).mean(dim=-1, keepdim=True)
    dx = gw * r - x * r.pow(3) * dot
    if grad_out is not None:
        dx = dx + _c(grad_out, compute)
    dweight = None if w is None else (g * x * r).reshape(-1, x.shape[-1]).sum(dim=0)
    return dx, dweight


# ---------------------------------------------------------------------------
# SwiGLU  (kernels.py:343-386, 690-700)
# ---------------------------------------------------------------------------
def swiglu(gate_up, compute=torch.float32):
    """silu(gate) * up with gate, up = gate_up.chunk(2, -1)   (kernels.py:351-358, 752-753)."""
    gate, up = _c(gate_up, compute).chunk(2, dim=-1)
    return F.silu(gate) * up


def swiglu_backward(gate_up, grad_out, compute=torch.float32):
    """dgate = g*up*s*(1+gate*(1-s)), dup = g*silu(gate)   (kernels.py:690-700)."""
    gate, up = _c(gate_up, compute).chunk(2, dim=-1)
    g = _c(grad_out, compute)
    s = torch.sigmoid(gate)
    return torch.cat((g * up * s * (1.0 + gate * (1.0 - s)), g * gate * s), dim=-1)


# ---------------------------------------------------------------------------
# RoPE tables and QK-norm + RoPE  (model.py:50-70; kernels.py:670-676, 703-735, 756-771)
# ---------------------------------------------------------------------------
def rope_tables(head_dim, seq_len, theta=1_000_000.0, fraction=0.25, dtype=torch.float32):
    """cos/sin [1, 1, T, rotary_dim] exactly as RotaryEmbedding builds them (model.py:50-70)."""
    rotary_dim = int(head_dim * fraction)
    rotary_dim -= rotary_dim % 2
    inv_freq = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2).float() / rotary_dim))
    t = torch.arange(seq_len, dtype=inv_freq.dtype)
    freqs = torch.outer(t, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos()[None, None].to(dtype), emb.sin()[None, None].to(dtype)


def apply_partial_rope(x, cos, sin):
    """Rotate-half on the first rotary_dim dims using cos/sin[..., :half]   (kernels.py:670-676)."""
    rotary_dim = cos.shape[-1]
    half = rotary_dim // 2
    c, s = cos[..., :half], sin[..., :half]
    x1, x2, xp = x[..., :half], x[..., half:rotary_dim], x[..., rotary_dim:]
    return torch.cat((x1 * c - x2 * s, x2 * c + x1 * s, xp), dim=-1)


def _orient(cos, sin, T):
    # accept [1,1,T,rd] or [1,T,1,rd]; return [1,T,1,rd]
    if cos.ndim == 4 and cos.shape[1] != T and cos.shape[2] == T:
        cos, sin = cos.transpose(1, 2), sin.transpose(1, 2)
    return cos, sin


def qk_norm_rope(q, k, cos, sin, eps=1e-6, compute=torch.float32):
    """rms_norm over head_dim then partial RoPE, q/k [B,T,H,D]   (kernels.py:766-771)."""
    cos, sin = _orient(_c(cos, compute), _c(sin, compute), q.shape[1])
    return (apply_partial_rope(rms_norm(q, None, eps, compute), cos, sin),
            apply_partial_rope(rms_norm(k, None, eps, compute), cos, sin))


def _norm_backward_no_weight(x, grad, eps):
    """(kernels.py:703-708)"""
    inv = torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
    dot = (grad * x).mean(dim=-1, keepdim=True)
    return grad * inv - x * inv.pow(3) * dot


def qk_norm_rope_backward(q, k, grad_q, grad_k, cos, sin, eps=1e-6, compute=torch.float32):
    """Inverse rotation of the gradient, then the weightless norm backward (kernels.py:732-734)."""
    cos, sin = _orient(_c(cos, compute), _c(sin, compute), q.shape[1])
    gq = apply_partial_rope(_c(grad_q, compute), cos, -sin)
    gk = apply_partial_rope(_c(grad_k, compute), cos, -sin)
    return (_norm_backward_no_weight(_c(q, compute), gq, eps),
            _norm_backward_no_weight(_c(k, compute), gk, eps))


def qkv_rope(x, w_qkv, cos, sin, n_head, n_kv_head, eps=1e-6, compute=torch.float32):
    """QKVProjection.fwd_torch: GEMM, split, view, QK-norm, RoPE   (model.py:92-115).

    Returns q, k, v in [B,T,H,D] (q, k normalised and rotated).
    """
    x = _c(x, compute)
    w = _c(w_qkv, compute)
    B, T, _ = x.shape
    D = w.shape[0] // (n_head + 2 * n_kv_head)
    qkv = x @ w.t()
    q, k, v = qkv.split((n_head * D, n_kv_head * D, n_kv_head * D), dim=-1)
    q = q.reshape(B, T, n_head, D)
    k = k.reshape(B, T, n_kv_head, D)
    v = v.reshape(B, T, n_kv_head, D)
    cos, sin = _orient(_c(cos, compute), _c(sin, compute), T)
    return (apply_partial_rope(rms_norm(q, None, eps, compute), cos, sin),
            apply_partial_rope(rms_norm(k, None, eps, compute), cos, sin), v)


def qkv_rope_backward(x, w_qkv, cos, sin, grad_q, grad_k, grad_v, n_head, n_kv_head, eps=1e-6,
                      compute=torch.float32):
    """(grad_x, grad_w) by autograd through qkv_rope's forward expression."""
    xr = _c(x, compute).detach().clone().requires_grad_(True)
    wr = _c(w_qkv, compute).detach().clone().requires_grad_(True)
    with torch.enable_grad():
        q, k, v = qkv_rope(xr, wr, cos, sin, n_head, n_kv_head, eps, compute)
        loss = ((q * _c(grad_q, compute)).sum() + (k * _c(grad_k, compute)).sum()
                + (v * _c(grad_v, compute)).sum())
        gx, gw = torch.autograd.grad(loss, (xr, wr))
    return gx, gw


# ---------------------------------------------------------------------------
# LM head + cross-entropy  (model.py:325-339; kernels.py:878-959)
# ---------------------------------------------------------------------------
def lm_head_ce(hidden, weight, targets, ignore_index=-100, chunk_size=4096, compute=torch.float32,
               need_grads=True):
    """Chunked logits + cross-entropy as LMHeadProjection.fwd_torch does (model.py:325-339).

    Loss = sum over chunks of CE_sum(logits, targets) / n, with rows whose
    target is ``ignore_index`` excluded and n = number of other rows (the
    F.cross_entropy ignore_index semantics; with no ignored row this is the
    reference's division by n_tokens).  Returns (loss, grad_hidden, grad_weight)
    with gradients from the closed form dlogits = (softmax - onehot)/n
    (kernels.py:315-318) and dX = dlogits @ W, dW = dlogits^T @ H
    (kernels.py:920-922).
    """
    h = _c(hidden, compute).reshape(-1, hidden.shape[-1])
    w = _c(weight, compute)
    t = targets.reshape(-1).to("cpu", torch.int64)
    valid = t != ignore_index
    n_valid = int(valid.sum())
    n = h.shape[0]
    chunk = chunk_size or n
    loss_sum = torch.zeros((), dtype=compute)
    gx = torch.zeros_like(h) if need_grads else None
    gw = torch.zeros_like(w) if need_grads else None
    for s in range(0, n, chunk):
        e = min(s + chunk, n)
        logits = h[s:e] @ w.t()
        tc = t[s:e]
        loss_sum = loss_sum + F.cross_entropy(logits, tc, ignore_index=ignore_index, reduction="sum")
        if need_grads:
            p = torch.softmax(logits, dim=-1)
            vm = valid[s:e]
            rows = torch.nonzero(vm).squeeze(-1)
            p[rows, tc[rows]] -= 1.0
            p[~vm] = 0.0
            p = p / max(n_valid, 1)
            gx[s:e] = p @ w
            gw += p.t() @ h[s:e]
    loss = loss_sum / n_valid if n_valid > 0 else torch.tensor(float("nan"), dtype=compute)
    return loss, gx, gw
