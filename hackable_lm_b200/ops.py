"""PyTorch custom operators over the libhlm_b200 C ABI.

Every operator here is a ``torch.library.custom_op`` in the
``hackable_lm_b200`` namespace with a fake (meta) implementation, so it stays
opaque and shape-correct under ``torch.compile(fullgraph=True)`` and CUDA
graph capture.  Outputs and workspaces are allocated by PyTorch's caching
allocator; the CUDA library itself never allocates, never synchronises, and
launches on the current stream of the tensor's device.

There is no CPU path: a CPU tensor raises.  The reference's CPU behaviour is
restated separately (test-only) for parity checking.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib
from ._lib import HLM_BF16, HLM_F16, HLM_F32, check

_DTYPE_CODE = {torch.float32: HLM_F32, torch.bfloat16: HLM_BF16, torch.float16: HLM_F16}


def _code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise RuntimeError(f"hackable_lm_b200: unsupported dtype {dtype}") from None


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    for t in tensors:
        if t.device.type != "cuda":
            raise RuntimeError(
                "hackable_lm_b200 operators run only on CUDA tensors (sm_100a); got a tensor on "
                f"{t.device}"
            )
        if t.device != dev:
            raise RuntimeError("hackable_lm_b200: all tensors must be on the same device")
    return dev


def _stream(dev: torch.device) -> int:
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if torch.cuda.current_device() != idx:
        torch.cuda.set_device(idx)
    return torch.cuda.current_stream(idx).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _lib_():
    return _lib.load()


# ---------------------------------------------------------------------------
# SwiGLU  (reference: kernels.py:343-419, 685-700, 743-753)
# ---------------------------------------------------------------------------
@torch.library.custom_op("hackable_lm_b200::swiglu", mutates_args=())
def swiglu(gate_up: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(gate_up)
    gate_up = gate_up.contiguous()
    hidden = gate_up.shape[-1] // 2
    rows = gate_up.numel() // max(1, 2 * hidden)
    out = torch.empty((*gate_up.shape[:-1], hidden), dtype=gate_up.dtype, device=dev)
    check(_lib_().hlm_swiglu_fwd(_ptr(gate_up), _ptr(out), rows, hidden, _code(gate_up.dtype),
                                  _stream(dev)), "hlm_swiglu_fwd")
    return out


@swiglu.register_fake
def _swiglu_fake(gate_up):
    return gate_up.new_empty((*gate_up.shape[:-1], gate_up.shape[-1] // 2))


@torch.library.custom_op("hackable_lm_b200::swiglu_backward", mutates_args=())
def swiglu_backward(gate_up: torch.Tensor, grad_out: torch.Tensor) -> torch.Tensor:
    dev = _require_cuda(gate_up, grad_out)
    gate_up = gate_up.contiguous()
    grad_out = grad_out.contiguous()
    hidden = grad_out.shape[-1]
    rows = grad_out.numel() // max(1, hidden)
    grad = torch.empty_like(gate_up)
    check(_lib_().hlm_swiglu_bwd(_ptr(gate_up), _ptr(grad_out), _ptr(grad), rows, hidden,
                                  _code(gate_up.dtype), _stream(dev)), "hlm_swiglu_bwd")
    return grad


@swiglu_backward.register_fake
def _swiglu_backward_fake(gate_up, grad_out):
    return torch.empty_like(gate_up)


def _swiglu_setup(ctx, inputs, output):
    (gate_up,) = inputs
    ctx.save_for_backward(gate_up)


def _swiglu_bwd(ctx, grad_out):
    if grad_out is None:
        return None
    (gate_up,) = ctx.saved_tensors
    return swiglu_backward(gate_up, grad_out)


swiglu.register_autograd(_swiglu_bwd, setup_context=_swiglu_setup)


def gate_up_swiglu_supported(x: torch.Tensor, weight: torch.Tensor) -> bool:
    """Shapes and dtypes the fused gate_up + SwiGLU kernel takes."""
    return ((x.is_cuda or x.is_meta) and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and x.shape[-1] % 64 == 0 and weight.shape[0] % 256 == 0 and weight.shape[1] == x.shape[-1])


# gate_up projection + SwiGLU (reference: model.py:285-292 -> kernels.py:743-753; its backward
# kernels.py:690-700 followed by the two weight-side GEMMs of the linear layer)
@torch.library.custom_op("hackable_lm_b200::gate_up_swiglu", mutates_args=())
def gate_up_swiglu(x: torch.Tensor, weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """h = silu(gate) * up with [gate | up] = x @ weight^T, in one tcgen05 GEMM.
    Returns (h [..., H], gate_up [..., 2H]); gate_up is kept for the backward."""
    dev = _require_cuda(x, weight)
    x = x.contiguous()
    weight = weight.contiguous()
    C = x.shape[-1]
    H = weight.shape[0] // 2
    rows = x.numel() // max(1, C)
    gate_up = torch.empty((*x.shape[:-1], 2 * H), dtype=x.dtype, device=dev)
    h = torch.empty((*x.shape[:-1], H), dtype=x.dtype, device=dev)
    check(_lib_().hlm_gate_up_swiglu_fwd(_ptr(x), _ptr(weight), _ptr(gate_up), _ptr(h), rows, C, H,
                                          _stream(dev)), "hlm_gate_up_swiglu_fwd")
    return h, gate_up


@gate_up_swiglu.register_fake
def _gate_up_swiglu_fake(x, weight):
    H = weight.shape[0] // 2
    return x.new_empty((*x.shape[:-1], H)), x.new_empty((*x.shape[:-1], 2 * H))


def _gate_up_setup(ctx, inputs, output):
    x, weight = inputs
    _, gate_up = output
    ctx.save_for_backward(x, weight, gate_up)
    # gate_up is differentiable so that swiglu_down can hand its gradient
    # straight to it; an output that receives no gradient arrives as None (no
    # zero-filled [M, 2H] tensor is materialised)
    ctx.set_materialize_grads(False)


def _gate_up_bwd(ctx, grad_h, grad_gate_up):
    x, weight, gate_up = ctx.saved_tensors
    dgu = None
    if grad_h is not None:
        dgu = swiglu_backward(gate_up, grad_h)
    if grad_gate_up is not None:
        dgu = grad_gate_up if dgu is None else dgu + grad_gate_up
    if dgu is None:
        return None, None
    C = x.shape[-1]
    d2 = dgu.reshape(-1, dgu.shape[-1])
    grad_x = (d2 @ weight).reshape(x.shape) if ctx.needs_input_grad[0] else None
    grad_w = (d2.t() @ x.reshape(-1, C)) if ctx.needs_input_grad[1] else None
    return grad_x, grad_w


gate_up_swiglu.register_autograd(_gate_up_bwd, setup_context=_gate_up_setup)


def swiglu_down_supported(w_gate_up: torch.Tensor, w_down: torch.Tensor) -> bool:
    """Shapes and dtypes of the fused down-projection backward (grad_h GEMM + SwiGLU backward)."""
    C, H = w_down.shape
    return ((w_down.is_cuda or w_down.is_meta) and w_down.dtype == torch.bfloat16 and w_gate_up.dtype == torch.bfloat16
            and C % 64 == 0 and H % 256 == 0 and w_gate_up.shape[0] == 2 * H)


# Down projection of h = swiglu(gate_up) (reference: model.py:295-304, the F.linear of
# DownProjection; its backward composed with _swiglu_backward, kernels.py:690-700)
@torch.library.custom_op("hackable_lm_b200::swiglu_down", mutates_args=())
def swiglu_down(h: torch.Tensor, gate_up: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """y = h @ weight^T, where h must be swiglu(gate_up) (the h and gate_up returned
    together by gate_up_swiglu).  The backward does not return a gradient for h:
    it sends the gradient through the SwiGLU to gate_up directly, computing
    grad_h = grad_y @ weight and the SwiGLU backward in one tcgen05 GEMM
    (grad_h never goes to memory); the weight gradient is grad_y^T @ h."""
    _require_cuda(h, gate_up, weight)
    return torch.nn.functional.linear(h, weight)


@swiglu_down.register_fake
def _swiglu_down_fake(h, gate_up, weight):
    return h.new_empty((*h.shape[:-1], weight.shape[0]))


def _swiglu_down_setup(ctx, inputs, output):
    h, gate_up, weight = inputs
    ctx.save_for_backward(h, gate_up, weight)
    ctx.set_materialize_grads(False)


def _swiglu_down_grad_into(grad_y: torch.Tensor, weight: torch.Tensor, gate_up: torch.Tensor,
                           out: torch.Tensor) -> None:
    dev = _require_cuda(grad_y, weight, gate_up, out)
    C, H = weight.shape
    gy = grad_y.contiguous()
    g = gate_up.contiguous()
    w = weight.contiguous()
    if not out.is_contiguous() or out.shape != g.shape or out.dtype != g.dtype:
        raise RuntimeError("swiglu_down_grad: out must be a contiguous tensor like gate_up")
    check(_lib_().hlm_swiglu_down_bwd(_ptr(gy), _ptr(w), _ptr(g), _ptr(out), gy.numel() // C, C, H,
                                       _stream(dev)), "hlm_swiglu_down_bwd")


@torch.library.custom_op("hackable_lm_b200::swiglu_down_backward", mutates_args=())
def swiglu_down_backward(grad_y: torch.Tensor, weight: torch.Tensor, gate_up: torch.Tensor) -> torch.Tensor:
    """grad_gate_up = swiglu_backward(gate_up, grad_y @ weight) in one kernel:
    grad_y [..., C], weight [C, H] (the down projection's nn.Linear weight), gate_up [..., 2H]."""
    out = torch.empty(gate_up.shape, dtype=gate_up.dtype, device=gate_up.device)
    _swiglu_down_grad_into(grad_y, weight, gate_up, out)
    return out


@swiglu_down_backward.register_fake
def _swiglu_down_backward_fake(grad_y, weight, gate_up):
    return torch.empty_like(gate_up, memory_format=torch.contiguous_format)


def swiglu_down_grad(grad_y: torch.Tensor, weight: torch.Tensor, gate_up: torch.Tensor,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """grad_gate_up = swiglu_backward(gate_up, grad_y @ weight) in one kernel (no autograd);
    with ``out`` given, written into it (the benchmark reuses one output buffer)."""
    if out is None:
        return swiglu_down_backward(grad_y, weight, gate_up)
    _swiglu_down_grad_into(grad_y, weight, gate_up, out)
    return out


def _swiglu_down_bwd(ctx, grad_y):
    h, gate_up, weight = ctx.saved_tensors
    if grad_y is None:
        return None, None, None
    C, H = weight.shape
    gy = grad_y.contiguous()
    grad_gate_up = None
    if ctx.needs_input_grad[0] or ctx.needs_input_grad[1]:
        grad_gate_up = swiglu_down_backward(gy, weight, gate_up)
    grad_w = None
    if ctx.needs_input_grad[2]:
        grad_w = gy.reshape(-1, C).t() @ h.reshape(-1, H)
    return None, grad_gate_up, grad_w


swiglu_down.register_autograd(_swiglu_down_bwd, setup_context=_swiglu_down_setup)


# ---------------------------------------------------------------------------
# Output / down projection + residual add + RMSNorm in one GEMM
# (reference: OutputProjection model.py:253-264, DownProjection model.py:295-304,
# residual_rms_norm model.py:73-75)
# ---------------------------------------------------------------------------
def proj_norm_supported(y: torch.Tensor, weight: torch.Tensor) -> bool:
    """Shapes the fused projection + residual + RMSNorm GEMM takes: bf16, K % 64 == 0,
    N = 1..4 x 256 or 1..4 x 128 (the row's N columns fit one thread-block cluster)."""
    N, K = weight.shape
    return ((y.is_cuda or y.is_meta) and y.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and y.shape[-1] == K and K % 64 == 0
            and ((N % 256 == 0 and N // 256 <= 4) or (N % 128 == 0 and N // 128 <= 4)))


def _proj_norm_fwd(y: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor,
                   eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(y, weight, residual)
    N, K = weight.shape
    y2 = y.contiguous()
    w = weight.contiguous()
    r = residual.contiguous()
    if r.shape[-1] != N or r.numel() // max(1, N) != y2.numel() // max(1, K) or r.dtype != y2.dtype:
        raise RuntimeError("proj_residual_norm: residual must be [..., N] with y's rows and dtype")
    out = torch.empty(r.shape, dtype=r.dtype, device=dev)
    norm = torch.empty(r.shape, dtype=r.dtype, device=dev)
    check(_lib_().hlm_proj_residual_rms_norm_fwd(_ptr(y2), _ptr(w), _ptr(r), _ptr(out), _ptr(norm),
                                                  y2.numel() // K, K, N, float(eps), _stream(dev)),
          "hlm_proj_residual_rms_norm_fwd")
    return out, norm


def _residual_norm_grad(out, grad_out, grad_norm, eps):
    """Gradient reaching residual + branch through out (directly and through the norm)."""
    if grad_norm is None:
        return grad_out
    g, _ = rms_norm_backward(out, None, grad_out, grad_norm, eps)
    return g


@torch.library.custom_op("hackable_lm_b200::proj_residual_norm", mutates_args=())
def proj_residual_norm(y: torch.Tensor, weight: torch.Tensor, residual: torch.Tensor,
                       eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """(out, norm) with out = residual + y @ weight^T and norm = rms_norm(out), one GEMM."""
    return _proj_norm_fwd(y, weight, residual, eps)


@proj_residual_norm.register_fake
def _proj_residual_norm_fake(y, weight, residual, eps):
    return (torch.empty_like(residual, memory_format=torch.contiguous_format),
            torch.empty_like(residual, memory_format=torch.contiguous_format))


def _proj_norm_setup(ctx, inputs, output):
    y, weight, residual, eps = inputs
    out, _ = output
    ctx.save_for_backward(y, weight, out)
    ctx.eps = eps
    ctx.set_materialize_grads(False)


def _proj_norm_bwd(ctx, grad_out, grad_norm):
    y, weight, out = ctx.saved_tensors
    if grad_out is None and grad_norm is None:
        return None, None, None, None
    g = _residual_norm_grad(out, grad_out, grad_norm, ctx.eps)
    N, K = weight.shape
    g2 = g.reshape(-1, N)
    grad_y = (g2 @ weight).reshape(y.shape) if ctx.needs_input_grad[0] else None
    grad_w = (g2.t() @ y.reshape(-1, K)) if ctx.needs_input_grad[1] else None
    return grad_y, grad_w, (g if ctx.needs_input_grad[2] else None), None


proj_residual_norm.register_autograd(_proj_norm_bwd, setup_context=_proj_norm_setup)


@torch.library.custom_op("hackable_lm_b200::swiglu_down_residual_norm", mutates_args=())
def swiglu_down_residual_norm(h: torch.Tensor, gate_up: torch.Tensor, weight: torch.Tensor,
                              residual: torch.Tensor, eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """The down projection of h = swiglu(gate_up) with the residual add and RMSNorm in its
    epilogue: (out, norm), out = residual + h @ weight^T.  Its backward sends the gradient
    of residual + branch through the fused grad_h GEMM + SwiGLU backward to gate_up (no
    gradient for h, as swiglu_down), and the weight gradient is g^T @ h."""
    return _proj_norm_fwd(h, weight, residual, eps)


@swiglu_down_residual_norm.register_fake
def _swiglu_down_residual_norm_fake(h, gate_up, weight, residual, eps):
    return (torch.empty_like(residual, memory_format=torch.contiguous_format),
            torch.empty_like(residual, memory_format=torch.contiguous_format))


def _sdrn_setup(ctx, inputs, output):
    h, gate_up, weight, residual, eps = inputs
    out, _ = output
    ctx.save_for_backward(h, gate_up, weight, out)
    ctx.eps = eps
    ctx.set_materialize_grads(False)


def _sdrn_bwd(ctx, grad_out, grad_norm):
    h, gate_up, weight, out = ctx.saved_tensors
    if grad_out is None and grad_norm is None:
        return None, None, None, None, None
    g = _residual_norm_grad(out, grad_out, grad_norm, ctx.eps)
    C, H = weight.shape
    gy = g.contiguous()
    grad_gate_up = None
    if ctx.needs_input_grad[0] or ctx.needs_input_grad[1]:
        grad_gate_up = swiglu_down_backward(gy, weight, gate_up)
    grad_w = (gy.reshape(-1, C).t() @ h.reshape(-1, H)) if ctx.needs_input_grad[2] else None
    return None, grad_gate_up, grad_w, (g if ctx.needs_input_grad[3] else None), None


swiglu_down_residual_norm.register_autograd(_sdrn_bwd, setup_context=_sdrn_setup)


# ---------------------------------------------------------------------------
# RMSNorm / residual-add + RMSNorm  (reference: model.py:14-16, 73-75; kernels.py:245-247)
# ---------------------------------------------------------------------------
def _rows_cols(x: torch.Tensor) -> tuple[int, int]:
    cols = x.shape[-1]
    return (x.numel() // cols if cols else 0), cols


@torch.library.custom_op("hackable_lm_b200::rms_norm", mutates_args=())
def rms_norm(x: torch.Tensor, weight: Optional[torch.Tensor], eps: float) -> torch.Tensor:
    dev = _require_cuda(x) if weight is None else _require_cuda(x, weight)
    x = x.contiguous()
    w = None if weight is None else weight.to(x.dtype).contiguous()
    rows, cols = _rows_cols(x)
    norm = torch.empty_like(x)
    check(_lib_().hlm_residual_rms_norm_fwd(None, _ptr(x), _ptr(w), None, _ptr(norm), rows, cols,
                                             float(eps), _code(x.dtype), _stream(dev)),
          "hlm_residual_rms_norm_fwd")
    return norm


@rms_norm.register_fake
def _rms_norm_fake(x, weight, eps):
    return torch.empty_like(x)


@torch.library.custom_op("hackable_lm_b200::residual_rms_norm", mutates_args=())
def residual_rms_norm(residual: torch.Tensor, branch: torch.Tensor, weight: Optional[torch.Tensor],
                      eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    tensors = [residual, branch] + ([] if weight is None else [weight])
    dev = _require_cuda(*tensors)
    if residual.shape != branch.shape or residual.dtype != branch.dtype:
        raise RuntimeError("residual_rms_norm: residual and branch must match in shape and dtype")
    residual = residual.contiguous()
    branch = branch.contiguous()
    w = None if weight is None else weight.to(branch.dtype).contiguous()
    rows, cols = _rows_cols(branch)
    out = torch.empty_like(branch)
    norm = torch.empty_like(branch)
    check(_lib_().hlm_residual_rms_norm_fwd(_ptr(residual), _ptr(branch), _ptr(w), _ptr(out),
                                             _ptr(norm), rows, cols, float(eps),
                                             _code(branch.dtype), _stream(dev)),
          "hlm_residual_rms_norm_fwd")
    return out, norm


@residual_rms_norm.register_fake
def _residual_rms_norm_fake(residual, branch, weight, eps):
    return torch.empty_like(branch), torch.empty_like(branch)


@torch.library.custom_op("hackable_lm_b200::rms_norm_backward", mutates_args=())
def rms_norm_backward(x: torch.Tensor, weight: Optional[torch.Tensor],
                      grad_out: Optional[torch.Tensor], grad_norm: torch.Tensor,
                      eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(x, grad_norm)
    x = x.contiguous()
    grad_norm = grad_norm.contiguous()
    go = None if grad_out is None else grad_out.contiguous()
    w = None if weight is None else weight.to(x.dtype).contiguous()
    rows, cols = _rows_cols(x)
    grad = torch.empty_like(x)
    if w is not None:
        gw = torch.empty(cols, dtype=x.dtype, device=dev)
        nbytes = _lib_().hlm_rms_norm_bwd_workspace_bytes(rows, cols)
        ws = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=dev)
    else:
        gw = torch.empty(0, dtype=x.dtype, device=dev)
        nbytes = 0
        ws = None
    check(_lib_().hlm_residual_rms_norm_bwd(_ptr(x), _ptr(w), _ptr(go), _ptr(grad_norm),
                                             _ptr(grad), _ptr(gw) if w is not None else None,
                                             _ptr(ws), nbytes, rows, cols, float(eps),
                                             _code(x.dtype), _stream(dev)),
          "hlm_residual_rms_norm_bwd")
    return grad, gw


@rms_norm_backward.register_fake
def _rms_norm_backward_fake(x, weight, grad_out, grad_norm, eps):
    cols = x.shape[-1]
    return torch.empty_like(x), x.new_empty(cols if weight is not None else 0)


def _rms_norm_setup(ctx, inputs, output):
    x, weight, eps = inputs
    ctx.save_for_backward(x, weight)
    ctx.eps = eps


def _rms_norm_bwd(ctx, grad_norm):
    x, weight = ctx.saved_tensors
    if grad_norm is None:
        return None, None, None
    gx, gw = rms_norm_backward(x, weight, None, grad_norm, ctx.eps)
    return gx, (gw.to(weight.dtype) if weight is not None else None), None


rms_norm.register_autograd(_rms_norm_bwd, setup_context=_rms_norm_setup)


def _residual_rms_norm_setup(ctx, inputs, output):
    residual, branch, weight, eps = inputs
    out, _ = output
    ctx.save_for_backward(out, weight)
    ctx.eps = eps


def _residual_rms_norm_bwd(ctx, grad_out, grad_norm):
    out, weight = ctx.saved_tensors
    if grad_norm is None:
        if grad_out is None:
            return None, None, None, None
        return grad_out, grad_out, (torch.zeros_like(weight) if weight is not None else None), None
    g, gw = rms_norm_backward(out, weight, grad_out, grad_norm, ctx.eps)
    return g, g, (gw.to(weight.dtype) if weight is not None else None), None


residual_rms_norm.register_autograd(_residual_rms_norm_bwd, setup_context=_residual_rms_norm_setup)


# ---------------------------------------------------------------------------
# QK-norm + RoPE  (reference: kernels.py:446-658, 679-682, 711-735, 756-771)
# ---------------------------------------------------------------------------
def _cos_sin_2d(cos: torch.Tensor, sin: torch.Tensor, seq_len: int) -> tuple[torch.Tensor, torch.Tensor, int]:
    rd = cos.shape[-1]
    c = cos.reshape(seq_len, rd)
    s = sin.reshape(seq_len, rd)
    if c.stride(1) != 1 or s.stride(1) != 1 or c.stride(0) != s.stride(0):
        c = c.contiguous()
        s = s.contiguous()
    return c, s, c.stride(0)


def _orient_cos(cos: torch.Tensor, sin: torch.Tensor, q: torch.Tensor):
    # Accept [1,1,T,rd] as well as [1,T,1,rd] (kernels.py:766-768).
    if cos.ndim == 4 and cos.shape[1] != q.shape[1] and cos.shape[2] == q.shape[1]:
        cos = cos.transpose(1, 2)
        sin = sin.transpose(1, 2)
    return cos, sin


@torch.library.custom_op("hackable_lm_b200::qk_norm_rope", mutates_args=())
def qk_norm_rope(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                 eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(q, k, cos, sin)
    B, T, Hq, D = q.shape
    Hk = k.shape[2]
    cos, sin = _orient_cos(cos, sin, q)
    rd = cos.shape[-1]
    c2, s2, cstride = _cos_sin_2d(cos, sin, T)
    q_out = torch.empty((B, T, Hq, D), dtype=q.dtype, device=dev)
    k_out = torch.empty((B, T, Hk, D), dtype=k.dtype, device=dev)
    check(_lib_().hlm_qk_norm_rope_fwd(
        _ptr(q), _ptr(k), _ptr(c2), _ptr(s2), _ptr(q_out), _ptr(k_out), B, T, Hq, Hk, D, rd,
        _lib.int64_array(q.stride()), _lib.int64_array(k.stride()), cstride, _code(c2.dtype),
        float(eps), _code(q.dtype), _stream(dev)), "hlm_qk_norm_rope_fwd")
    return q_out, k_out


@qk_norm_rope.register_fake
def _qk_norm_rope_fake(q, k, cos, sin, eps):
    return q.new_empty(q.shape), k.new_empty(k.shape)


@torch.library.custom_op("hackable_lm_b200::qk_norm_rope_backward", mutates_args=())
def qk_norm_rope_backward(q: torch.Tensor, k: torch.Tensor, grad_q: torch.Tensor,
                          grad_k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                          eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(q, k, grad_q, grad_k, cos, sin)
    B, T, Hq, D = q.shape
    Hk = k.shape[2]
    cos, sin = _orient_cos(cos, sin, q)
    rd = cos.shape[-1]
    c2, s2, cstride = _cos_sin_2d(cos, sin, T)
    grad_q = grad_q.contiguous()
    grad_k = grad_k.contiguous()
    gq = torch.empty((B, T, Hq, D), dtype=q.dtype, device=dev)
    gk = torch.empty((B, T, Hk, D), dtype=k.dtype, device=dev)
    check(_lib_().hlm_qk_norm_rope_bwd(
        _ptr(q), _ptr(k), _ptr(grad_q), _ptr(grad_k), _ptr(c2), _ptr(s2), _ptr(gq), _ptr(gk),
        B, T, Hq, Hk, D, rd, _lib.int64_array(q.stride()), _lib.int64_array(k.stride()), cstride,
        _code(c2.dtype), float(eps), _code(q.dtype), _stream(dev)), "hlm_qk_norm_rope_bwd")
    return gq, gk


@qk_norm_rope_backward.register_fake
def _qk_norm_rope_backward_fake(q, k, grad_q, grad_k, cos, sin, eps):
    return q.new_empty(q.shape), k.new_empty(k.shape)


def _qk_setup(ctx, inputs, output):
    q, k, cos, sin, eps = inputs
    ctx.save_for_backward(q, k, cos, sin)
    ctx.eps = eps


def _qk_bwd(ctx, grad_q, grad_k):
    q, k, cos, sin = ctx.saved_tensors
    if grad_q is None:
        grad_q = torch.zeros(q.shape, dtype=q.dtype, device=q.device)
    if grad_k is None:
        grad_k = torch.zeros(k.shape, dtype=k.dtype, device=k.device)
    gq, gk = qk_norm_rope_backward(q, k, grad_q, grad_k, cos, sin, ctx.eps)
    return gq, gk, None, None, None


qk_norm_rope.register_autograd(_qk_bwd, setup_context=_qk_setup)


# ---------------------------------------------------------------------------
# Fused QKV projection + QK-norm + RoPE  (reference: model.py:78-126)
# ---------------------------------------------------------------------------
FUSED_QKV_ROTARY_DIMS = (0, 16, 32, 64, 128)
FUSED_QKV_HEAD_DIM = 128


def fused_qkv_supported(head_dim: int, rotary_dim: int, n_embd: int) -> bool:
    return head_dim == FUSED_QKV_HEAD_DIM and rotary_dim in FUSED_QKV_ROTARY_DIMS and n_embd % 64 == 0


@torch.library.custom_op("hackable_lm_b200::qkv_rope", mutates_args=())
def qkv_rope(x: torch.Tensor, w_qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
             n_head: int, n_kv_head: int, eps: float
             ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    dev = _require_cuda(x, w_qkv, cos, sin)
    if x.dtype != torch.bfloat16 or w_qkv.dtype != torch.bfloat16:
        raise RuntimeError("qkv_rope: x and w_qkv must be bfloat16")
    B, T, C = x.shape
    D = w_qkv.shape[0] // (n_head + 2 * n_kv_head)
    rd = cos.shape[-1]
    c2, s2, cstride = _cos_sin_2d(cos, sin, T)
    x = x.contiguous()
    w = w_qkv.contiguous()
    q = torch.empty((B, T, n_head, D), dtype=x.dtype, device=dev)
    k = torch.empty((B, T, n_kv_head, D), dtype=x.dtype, device=dev)
    v = torch.empty((B, T, n_kv_head, D), dtype=x.dtype, device=dev)
    rstd = torch.empty((B * T, n_head + n_kv_head), dtype=torch.float32, device=dev)
    check(_lib_().hlm_qkv_rope_fwd(
        _ptr(x), _ptr(w), _ptr(c2), _ptr(s2), _ptr(q), _ptr(k), _ptr(v), _ptr(rstd), B, T, C,
        n_head, n_kv_head, D, rd, cstride, _code(c2.dtype), float(eps), _stream(dev)),
        "hlm_qkv_rope_fwd")
    return q, k, v, rstd


@qkv_rope.register_fake
def _qkv_rope_fake(x, w_qkv, cos, sin, n_head, n_kv_head, eps):
    B, T, C = x.shape
    D = w_qkv.shape[0] // (n_head + 2 * n_kv_head)
    return (x.new_empty((B, T, n_head, D)), x.new_empty((B, T, n_kv_head, D)),
            x.new_empty((B, T, n_kv_head, D)),
            x.new_empty((B * T, n_head + n_kv_head), dtype=torch.float32))


@torch.library.custom_op("hackable_lm_b200::qkv_rope_backward", mutates_args=())
def qkv_rope_backward(x: torch.Tensor, w_qkv: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
                      rstd: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                      grad_q: torch.Tensor, grad_k: torch.Tensor, grad_v: torch.Tensor,
                      n_head: int, n_kv_head: int, eps: float, need_dx: bool, need_dw: bool
                      ) -> tuple[torch.Tensor, torch.Tensor]:
    dev = _require_cuda(x, w_qkv, q, k, rstd, grad_q, grad_k, grad_v)
    B, T, C = x.shape
    D = q.shape[-1]
    rd = cos.shape[-1]
    c2, s2, cstride = _cos_sin_2d(cos, sin, T)
    grad_q = grad_q.contiguous()
    grad_k = grad_k.contiguous()
    grad_v = grad_v.contiguous()
    gx = torch.empty_like(x) if need_dx else x.new_empty(0)
    gw = torch.empty_like(w_qkv) if need_dw else w_qkv.new_empty(0)
    nbytes = _lib_().hlm_qkv_rope_bwd_workspace_bytes(B, T, C, n_head, n_kv_head, D)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    check(_lib_().hlm_qkv_rope_bwd(
        _ptr(x.contiguous()), _ptr(w_qkv.contiguous()), _ptr(q), _ptr(k), _ptr(rstd), _ptr(c2),
        _ptr(s2), _ptr(grad_q), _ptr(grad_k), _ptr(grad_v), _ptr(gx) if need_dx else None,
        _ptr(gw) if need_dw else None, _ptr(ws), nbytes, B, T, C, n_head, n_kv_head, D, rd,
        cstride, _code(c2.dtype), float(eps), _stream(dev)), "hlm_qkv_rope_bwd")
    return gx, gw


@qkv_rope_backward.register_fake
def _qkv_rope_backward_fake(x, w_qkv, q, k, rstd, cos, sin, grad_q, grad_k, grad_v, n_head,
                            n_kv_head, eps, need_dx, need_dw):
    return (torch.empty_like(x) if need_dx else x.new_empty(0),
            torch.empty_like(w_qkv) if need_dw else w_qkv.new_empty(0))


def _qkv_setup(ctx, inputs, output):
    x, w_qkv, cos, sin, n_head, n_kv_head, eps = inputs
    q, k, v, rstd = output
    ctx.save_for_backward(x, w_qkv, q, k, rstd, cos, sin)
    ctx.n_head = n_head
    ctx.n_kv_head = n_kv_head
    ctx.eps = eps


def _qkv_bwd(ctx, grad_q, grad_k, grad_v, grad_rstd):
    x, w_qkv, q, k, rstd, cos, sin = ctx.saved_tensors
    need_dx, need_dw = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
    if not (need_dx or need_dw):
        return None, None, None, None, None, None, None
    if grad_q is None:
        grad_q = torch.zeros_like(q)
    if grad_k is None:
        grad_k = torch.zeros_like(k)
    if grad_v is None:
        grad_v = torch.zeros(k.shape, dtype=k.dtype, device=k.device)
    gx, gw = qkv_rope_backward(x, w_qkv, q, k, rstd, cos, sin, grad_q, grad_k, grad_v,
                               ctx.n_head, ctx.n_kv_head, ctx.eps, need_dx, need_dw)
    return (gx if need_dx else None), (gw if need_dw else None), None, None, None, None, None


qkv_rope.register_autograd(_qkv_bwd, setup_context=_qkv_setup)


# ---------------------------------------------------------------------------
# Fused LM head + cross-entropy  (reference: kernels.py:872-959)
# ---------------------------------------------------------------------------
@torch.library.custom_op("hackable_lm_b200::lm_head_ce", mutates_args=())
def lm_head_ce(hidden: torch.Tensor, weight: torch.Tensor, targets: torch.Tensor,
               ignore_index: int, chunk_tokens: int, need_dx: bool, need_dw: bool
               ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    dev = _require_cuda(hidden, weight, targets)
    if hidden.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16:
        raise RuntimeError("lm_head_ce: hidden and weight must be bfloat16")
    hidden = hidden.contiguous()
    weight = weight.contiguous()
    targets = targets.to(torch.int64).contiguous()
    n, C = hidden.shape
    V = weight.shape[0]
    loss = torch.empty((), dtype=torch.float32, device=dev)
    gx = torch.empty_like(hidden) if need_dx else hidden.new_empty(0)
    gw = torch.empty_like(weight) if need_dw else weight.new_empty(0)
    nbytes = _lib_().hlm_lm_head_ce_workspace_bytes(n, C, V, chunk_tokens)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    check(_lib_().hlm_lm_head_ce(
        _ptr(hidden), _ptr(weight), _ptr(targets), _ptr(loss), _ptr(gx) if need_dx else None,
        _ptr(gw) if need_dw else None, _ptr(ws), nbytes, n, C, V, int(ignore_index),
        int(chunk_tokens), _stream(dev)), "hlm_lm_head_ce")
    return loss, gx, gw


@lm_head_ce.register_fake
def _lm_head_ce_fake(hidden, weight, targets, ignore_index, chunk_tokens, need_dx, need_dw):
    return (hidden.new_empty((), dtype=torch.float32),
            torch.empty_like(hidden) if need_dx else hidden.new_empty(0),
            torch.empty_like(weight) if need_dw else weight.new_empty(0))


@torch.library.custom_op("hackable_lm_b200::scale_", mutates_args=("x",))
def scale_(x: torch.Tensor, scale: torch.Tensor) -> None:
    dev = _require_cuda(x, scale)
    if not x.is_contiguous():
        raise RuntimeError("scale_: tensor must be contiguous")
    s = scale.to(torch.float32).contiguous()
    check(_lib_().hlm_scale_by_device_scalar(_ptr(x), _ptr(s), x.numel(), _code(x.dtype),
                                              _stream(dev)), "hlm_scale_by_device_scalar")


@scale_.register_fake
def _scale_fake(x, scale):
    return None


# ---------------------------------------------------------------------------
# Attention core: tcgen05 forward; tcgen05 (windows) or cuDNN backward  (reference: kernels.py:774-847)
# ---------------------------------------------------------------------------
def attention_supported(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    """[B, T, H, 128] bf16 q with k, v of the same heads, T a multiple of 128."""
    return ((q.is_cuda or q.is_meta) and q.dtype == torch.bfloat16 and q.dim() == 4 and q.shape[-1] == 128
            and q.shape[1] % 128 == 0 and k.shape == q.shape and v.shape == q.shape
            and k.dtype == q.dtype and v.dtype == q.dtype)


@torch.library.custom_op("hackable_lm_b200::attention", mutates_args=())
def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window: int,
              scale: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Causal attention on [B, T, H, 128] bf16 (keys with 0 <= t - k < window; window <= 0
    means full causal).  Returns (out [B, T, H, 128], lse [B, H, T] fp32, natural log)."""
    dev = _require_cuda(q, k, v)
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    B, T, H, D = q.shape
    Hk = k.shape[2]
    out = torch.empty_like(q)
    lse = torch.empty((B, H, T), dtype=torch.float32, device=dev)
    check(_lib_().hlm_attention_fwd(_ptr(q), _ptr(k), _ptr(v), _ptr(out), _ptr(lse), B, T, H, Hk, D,
                                     int(window), float(scale), _stream(dev)), "hlm_attention_fwd")
    return out, lse


@attention.register_fake
def _attention_fake(q, k, v, window, scale):
    B, T, H, _ = q.shape
    return torch.empty_like(q, memory_format=torch.contiguous_format), q.new_empty((B, H, T), dtype=torch.float32)


_FLASH_BWD = []

# Which backward attention_backward runs: "native" (hlm_attention_bwd, this
# library's tcgen05 kernel), "library" (cuDNN / flash_attn), or "auto": native for
# a sliding window (measured at [16, 2048, 6, 128], window 512: 311 us vs 540 us for
# flash_attn's windowed backward), cuDNN for full causal attention (335 us vs 455 us).
ATTENTION_BWD = {"mode": "auto"}


def _native_attention_bwd(window: int, T: int, H: int, Hk: int) -> bool:
    mode = ATTENTION_BWD["mode"]
    if H != Hk:
        return False
    if mode == "native":
        return True
    if mode == "library":
        return False
    return 0 < window < T


def _flash_attn_backward_op():
    """flash_attn's backward (library code, like cuBLAS for the plain GEMMs), which
    has a sliding-window kernel and takes the forward's output and natural-log lse
    in this layout; None when the package is not installed."""
    if not _FLASH_BWD:
        try:
            from flash_attn.flash_attn_interface import _flash_attn_backward
        except Exception:  # noqa: BLE001 - any import failure means "not available"
            _flash_attn_backward = None
        _FLASH_BWD.append(_flash_attn_backward)
    return _FLASH_BWD[0]


def _window_bias(T: int, window: int, device) -> torch.Tensor:
    pos = torch.arange(T, device=device)
    dist = pos[:, None] - pos[None, :]
    keep = (dist >= 0) & (dist < window)
    return torch.zeros((T, T), dtype=torch.bfloat16, device=device).masked_fill(~keep, float("-inf"))


@torch.library.custom_op("hackable_lm_b200::attention_backward", mutates_args=())
def attention_backward(grad_out: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                       out: torch.Tensor, lse: torch.Tensor, window: int,
                       scale: float) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Gradients of attention(), fed with its output and log-sum-exp: for a sliding
    window this library's tcgen05 backward (hlm_attention_bwd); for full causal
    attention cuDNN's SDPA backward (library code, as cuBLAS is for the plain GEMMs,
    and faster there today); ATTENTION_BWD selects.  Without the native kernel (grouped
    heads, or mode "library") a window goes to flash_attn's windowed backward, or to
    cuDNN with the window as a dense T x T bias when flash_attn is not installed
    (measured at [16, 2048, 6, 128], window 512: native 0.31 ms, flash_attn 0.54 ms,
    cuDNN with the bias 1.3 ms)."""
    _require_cuda(grad_out, q, k, v, out, lse)
    B, T, H, D = q.shape
    full = window <= 0 or window >= T
    if _native_attention_bwd(window, T, H, k.shape[2]):
        dev = q.device
        q, k, v, out = q.contiguous(), k.contiguous(), v.contiguous(), out.contiguous()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        lib = _lib_()
        nbytes = int(lib.hlm_attention_bwd_workspace_bytes(B, T, H, D))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        check(lib.hlm_attention_bwd(_ptr(grad_out.contiguous()), _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                                    _ptr(lse.contiguous()), _ptr(dq), _ptr(dk), _ptr(dv), _ptr(ws), nbytes,
                                    B, T, H, k.shape[2], D, int(window), float(scale), _stream(dev)),
              "hlm_attention_bwd")
        return dq, dk, dv
    fa_bwd = None if full else _flash_attn_backward_op()
    if fa_bwd is not None:
        q, k, v, out = q.contiguous(), k.contiguous(), v.contiguous(), out.contiguous()
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
        # keys with 0 <= t - k < window: causal, left window window - 1, no dropout
        fa_bwd(grad_out.contiguous(), q, k, v, out, lse.contiguous(), dq, dk, dv, 0.0, float(scale), True,
               int(window) - 1, 0, 0.0, None, False, None)
        return dq, dk, dv
    # [B, H, T, D] views of the [B, T, H, D] tensors: q, k, v, out and grad_out share
    # one stride pattern, as cuDNN's backward expects of tensors from its own forward;
    # no dropout (seed / offset zero), dense (no cumulative sequence lengths), the
    # log-sum-exp as its [B, H, T, 1] statistics
    tr = lambda t: t.transpose(1, 2)  # noqa: E731
    zero = torch.zeros((), dtype=torch.int64, device=q.device)
    bias = None if full else _window_bias(T, window, q.device)[None, None].expand(B, H, T, T)
    dq, dk, dv = torch.ops.aten._scaled_dot_product_cudnn_attention_backward(
        tr(grad_out.contiguous()), tr(q), tr(k), tr(v), tr(out), lse.unsqueeze(-1), zero, zero, bias, None, None,
        T, T, 0.0, full, scale=scale)
    return dq.transpose(1, 2).contiguous(), dk.transpose(1, 2).contiguous(), dv.transpose(1, 2).contiguous()


@attention_backward.register_fake
def _attention_backward_fake(grad_out, q, k, v, out, lse, window, scale):
    return torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)


def _attention_setup(ctx, inputs, output):
    q, k, v, window, scale = inputs
    out, lse = output
    ctx.save_for_backward(q, k, v, out, lse)
    ctx.window = window
    ctx.scale = scale
    ctx.set_materialize_grads(False)


def _attention_bwd(ctx, grad_out, grad_lse):
    q, k, v, out, lse = ctx.saved_tensors
    if grad_out is None:
        return None, None, None, None, None
    dq, dk, dv = attention_backward(grad_out, q, k, v, out, lse, ctx.window, ctx.scale)
    return dq, dk, dv, None, None


attention.register_autograd(_attention_bwd, setup_context=_attention_setup)


# ---------------------------------------------------------------------------
# Plain tcgen05 GEMM (building block, used by tests and the bench)
# ---------------------------------------------------------------------------
def gemm(a: torch.Tensor, b: torch.Tensor, *, a_mn_major: bool = False, b_mn_major: bool = False,
         out: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.bfloat16,
         accumulate: bool = False) -> torch.Tensor:
    """D = A @ B^T on the tensor cores.

    a: [M, K] (or [K, M] with a_mn_major), b: [N, K] (or [K, N] with b_mn_major),
    both bf16 row-major contiguous.  Returns D [M, N] in out_dtype (bf16/fp32).
    """
    dev = _require_cuda(a, b)
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
        raise RuntimeError("gemm: operands must be bfloat16")
    a = a.contiguous()
    b = b.contiguous()
    M, K = (a.shape[1], a.shape[0]) if a_mn_major else (a.shape[0], a.shape[1])
    N = b.shape[1] if b_mn_major else b.shape[0]
    Kb = b.shape[0] if b_mn_major else b.shape[1]
    if K != Kb:
        raise RuntimeError(f"gemm: K mismatch {K} vs {Kb}")
    if out is None:
        out = torch.empty((M, N), dtype=out_dtype, device=dev)
    check(_lib_().hlm_gemm_bf16(
        _ptr(a), _ptr(b), _ptr(out), M, N, K, int(a_mn_major), int(b_mn_major), a.shape[1],
        b.shape[1], out.stride(0), _code(out.dtype), int(accumulate), _stream(dev)),
        "hlm_gemm_bf16")
    return out
