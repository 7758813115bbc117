"""Drop-in operator layer: the reference ``kernels.py`` entry points on sm_100a.

The functions that hackable-lm's ``model.py`` and ``train.py`` call keep their
names and signatures (kernels.py:126-972 in the reference), and route to the
hand-written CUDA kernels of ``libhlm_b200.so`` through the custom operators in
:mod:`hackable_lm_b200.ops`:

=====================================  =========================================
reference entry point                  B200 implementation
=====================================  =========================================
``swiglu_triton(gate_up)``             ``hackable_lm_b200::swiglu`` (+ backward)
``qk_norm_rope_triton(q,k,cos,sin,e)`` ``hackable_lm_b200::qk_norm_rope``
``fused_linear_cross_entropy_with_``   ``hackable_lm_b200::lm_head_ce`` (tcgen05
``weight(h, W, bias, t, backend, c)``  logits GEMM + online LSE + dX/dW GEMMs)
``rms_norm(x, weight, eps)``           ``hackable_lm_b200::rms_norm``
``model.residual_rms_norm(r, b, eps)`` ``hackable_lm_b200::residual_rms_norm``
=====================================  =========================================

The module backend value ``"triton"`` is accepted as an alias of ``"b200"`` so
that reference configs and command lines select the new path unchanged.  The
new path has no CPU fallback: CPU tensors raise.
"""
from __future__ import annotations

import math
from dataclasses import asdict, dataclass
from typing import Any

import torch
import torch.nn.functional as F

from . import ops
from .config import MODULE_BACKEND_FIELDS, MODULE_BACKENDS, normalize_attention_backend

B200_MODULE_BACKENDS = frozenset(MODULE_BACKEND_FIELDS)
# Reference name kept for callers that import it (kernels.py:49-53); on this
# path every module backend field has a B200 implementation.
TRITON_MODULE_BACKENDS = B200_MODULE_BACKENDS


@dataclass
class KernelInfo:
    requested_backend: str
    attention_backend: str
    qkv_backend: str
    output_backend: str
    gate_up_backend: str
    down_backend: str
    lm_head_backend: str
    torch_compile: bool
    torch_compile_mode: str
    torch_compile_capture_scalar_outputs: bool
    precision: str
    b200_library: str
    b200_library_version: int

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def _cuda_only(t: torch.Tensor, what: str) -> None:
    # meta tensors carry shapes only: they reach the operators' fake
    # implementations (shape propagation, meta-device model construction), never a kernel
    if not (t.is_cuda or t.is_meta):
        raise RuntimeError(
            f"{what}: the hackable_lm_b200 path runs only on CUDA (sm_100a) tensors; "
            "use the 'torch' module backend for CPU runs"
        )


def resolve_kernel_backends(
    requested: str,
    precision: str,
    compile_model: bool,
    compile_mode: str = "default",
    compile_capture_scalar_outputs: bool = True,
    attention_backend: str = "sdpa",
    allow_torch_backend: bool = False,
    **module_backends: str,
) -> KernelInfo:
    """Validate backend names the way the reference does (kernels.py:146-242).

    Module backends resolve to ``"torch"`` or ``"b200"`` (``"triton"`` is an
    alias of ``"b200"``).  Requesting ``"b200"`` loads the CUDA library and
    fails loudly if it is missing.
    """
    from . import _lib

    requested = requested.lower()
    if requested != "torch":
        raise ValueError(f"unknown kernel backend {requested!r}")
    unknown = set(module_backends) - set(MODULE_BACKEND_FIELDS)
    if unknown:
        raise ValueError(f"unknown module backend fields {sorted(unknown)!r}")
    resolved = {}
    for name in MODULE_BACKEND_FIELDS:
        value = module_backends.get(name, "torch")
        if not isinstance(value, str):
            raise ValueError(f"unknown {name} {value!r}")
        backend = value.lower()
        if backend not in MODULE_BACKENDS:
            raise ValueError(f"unknown {name} {backend!r}")
        resolved[name] = "b200" if backend == "triton" else backend
    attention = normalize_attention_backend(attention_backend)
    if precision != "bf16" and not allow_torch_backend:
        raise RuntimeError(f"unsupported precision mode {precision!r}; the training fast path uses bf16")
    lib_version = 0
    lib_path = str(_lib.LIB_PATH)
    if any(v == "b200" for v in resolved.values()):
        lib_version = int(_lib.load().hlm_version())
    return KernelInfo(
        requested_backend=requested,
        attention_backend=attention,
        **resolved,
        torch_compile=compile_model,
        torch_compile_mode=compile_mode,
        torch_compile_capture_scalar_outputs=compile_capture_scalar_outputs,
        precision=precision,
        b200_library=lib_path,
        b200_library_version=lib_version,
    )


def compile_training_model(model: torch.nn.Module, enabled: bool, mode: str = "default",
                           capture_scalar_outputs: bool = True) -> torch.nn.Module:
    """torch.compile wrapper with the reference's settings (kernels.py:126-137)."""
    if not enabled:
        return model
    import torch._dynamo

    torch._dynamo.config.capture_scalar_outputs = capture_scalar_outputs
    return torch.compile(model, mode=None if mode == "default" else mode, dynamic=False, fullgraph=True)


def mark_compiled_step_begin(enabled: bool) -> None:
    if enabled:
        torch.compiler.cudagraph_mark_step_begin()


# ---------------------------------------------------------------------------
# Hot-path entry points
# ---------------------------------------------------------------------------
def rms_norm(x: torch.Tensor, weight: torch.Tensor | None, eps: float) -> torch.Tensor:
    """x * rsqrt(mean(x^2) + eps) [* weight]  (kernels.py:245-247)."""
    _cuda_only(x, "rms_norm")
    return ops.rms_norm(x, weight, eps)


def residual_rms_norm(residual: torch.Tensor, branch: torch.Tensor, eps: float,
                      weight: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """(residual + branch, rms_norm(residual + branch))  (model.py:73-75)."""
    _cuda_only(branch, "residual_rms_norm")
    return ops.residual_rms_norm(residual, branch, weight, eps)


def swiglu_triton(gate_up: torch.Tensor) -> torch.Tensor:
    """silu(gate) * up on the packed [..., 2H] projection (kernels.py:743-753)."""
    if gate_up.shape[-1] % 2:
        raise RuntimeError(f"SwiGLU input last dimension must be even, got {gate_up.shape[-1]}")
    _cuda_only(gate_up, "swiglu")
    return ops.swiglu(gate_up)


def qk_norm_rope_triton(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                        eps: float) -> tuple[torch.Tensor, torch.Tensor]:
    """Weightless RMSNorm over head_dim, then partial rotate-half RoPE (kernels.py:756-771)."""
    _cuda_only(q, "qk_norm_rope")
    if cos.shape[-1] % 2:
        raise RuntimeError(f"rotary dim must be even, got {cos.shape[-1]}")
    return ops.qk_norm_rope(q, k, cos, sin, eps)


def qkv_projection_rope(x: torch.Tensor, w_qkv: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                        n_head: int, n_kv_head: int, eps: float
                        ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Fused x @ w_qkv^T + head split + QK-norm + RoPE (QKVProjection, model.py:92-126).

    Runs as one tcgen05 GEMM with the norm/RoPE in its epilogue when
    head_dim == 128, rotary_dim is 0/16/32/64/128 and cos/sin are bf16 or fp32;
    otherwise as the reference structure (nn.Linear GEMM, strided split) feeding
    the standalone qk_norm_rope kernel.
    """
    _cuda_only(x, "qkv_projection_rope")
    B, T, C = x.shape
    head_dim = w_qkv.shape[0] // (n_head + 2 * n_kv_head)
    rd = cos.shape[-1]
    if (ops.fused_qkv_supported(head_dim, rd, C) and x.dtype == torch.bfloat16
            and cos.dtype in (torch.bfloat16, torch.float32)):
        q, k, v, _ = ops.qkv_rope(x, w_qkv, cos, sin, n_head, n_kv_head, eps)
        return q, k, v
    qkv = F.linear(x, w_qkv)
    q_dim, kv_dim = n_head * head_dim, n_kv_head * head_dim
    q, k, v = qkv.split((q_dim, kv_dim, kv_dim), dim=-1)
    q = q.view(B, T, n_head, head_dim)
    k = k.view(B, T, n_kv_head, head_dim)
    v = v.view(B, T, n_kv_head, head_dim)
    q, k = ops.qk_norm_rope(q, k, cos.reshape(1, T, 1, rd), sin.reshape(1, T, 1, rd), eps)
    return q, k, v


class _B200FusedLinearCrossEntropy(torch.autograd.Function):
    """Forward computes loss, dX and dW in one library call; backward only
    rescales the saved gradients by grad_output (kernels.py:878-942)."""

    @staticmethod
    def forward(ctx, hidden, weight, targets, ignore_index, requested_chunk_size):
        if requested_chunk_size is not None and requested_chunk_size < 0:
            raise RuntimeError(f"loss_chunk_size must be nonnegative, got {requested_chunk_size}")
        need_dx = hidden.requires_grad
        need_dw = weight.requires_grad
        loss, gx, gw = ops.lm_head_ce(hidden, weight, targets, int(ignore_index), 0, need_dx, need_dw)
        ctx.save_for_backward(gx if need_dx else None, gw if need_dw else None)
        ctx.need = (need_dx, need_dw)
        return loss

    @staticmethod
    def backward(ctx, grad_output):
        gx, gw = ctx.saved_tensors
        need_dx, need_dw = ctx.need
        if need_dx and ctx.needs_input_grad[0]:
            ops.scale_(gx, grad_output)
        else:
            gx = None
        if need_dw and ctx.needs_input_grad[1]:
            ops.scale_(gw, grad_output)
        else:
            gw = None
        return gx, gw, None, None, None


def fused_linear_cross_entropy_with_weight(hidden: torch.Tensor, weight: torch.Tensor,
                                           bias: torch.Tensor | None, targets: torch.Tensor,
                                           backend: str, chunk_size: int | None = None,
                                           ignore_index: int = -100) -> torch.Tensor:
    """Mean cross-entropy of hidden @ weight^T against targets (kernels.py:945-959).

    Rows whose target equals ``ignore_index`` contribute neither loss nor
    gradient, and the mean runs over the remaining rows (F.cross_entropy
    semantics).  ``chunk_size`` is validated as in the reference; the library
    sizes its own token chunks from a memory budget, which changes only the
    order of floating-point accumulation, not the result.
    """
    if backend not in {"triton", "b200"}:
        raise RuntimeError(f"unsupported fused linear cross entropy backend {backend!r}")
    if bias is not None:
        raise RuntimeError("the B200 fused LM head has no bias term (the model uses bias=False)")
    hidden_flat = hidden.reshape(-1, hidden.size(-1))
    targets_flat = targets.reshape(-1).contiguous()
    _cuda_only(hidden_flat, "fused_linear_cross_entropy")
    return _B200FusedLinearCrossEntropy.apply(hidden_flat, weight, targets_flat, ignore_index, chunk_size)


@dataclass(frozen=True)
class WindowBlockMask:
    """What ``flex_attention_block_mask`` returns on this path: the causal
    (optionally sliding-window) pattern the reference encodes in a FlexAttention
    BlockMask (kernels.py:850-869), kept as its two parameters so that the
    attention core can run it on SDPA."""

    seq_len: int
    window_size: int | None


def flex_attention_block_mask(batch_size: int, n_head: int, seq_len: int, device: torch.device,
                              window_size: int | None = None) -> WindowBlockMask:
    """Reference signature (kernels.py:850-856): causal mask, plus
    ``q - kv < window_size`` when a window is given."""
    del batch_size, n_head, device
    return WindowBlockMask(int(seq_len), None if window_size is None else int(window_size))


def _sdpa_core(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, dropout_p: float, is_causal: bool,
               attn_mask: torch.Tensor | None, window_size: int | None) -> torch.Tensor:
    """torch SDPA on [B, H, T, D]; a sliding window becomes the boolean mask
    ``0 <= q - kv < window`` (the FlashAttention window ``(window - 1, 0)`` of
    kernels.py:839 and the reference's own mask, model.py:143-153)."""
    if window_size is not None and attn_mask is None:
        T = q.shape[-2]
        pos = torch.arange(T, device=q.device)
        dist = pos[:, None] - pos[None, :]
        attn_mask = (dist >= 0) & (dist < window_size)
        is_causal = False
    return F.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, dropout_p=dropout_p,
                                          is_causal=is_causal and attn_mask is None,
                                          enable_gqa=q.shape[1] != k.shape[1])


_FLASH_BACKENDS = ("flash_attn_2", "flash_attn_3", "flash_attn_4")


def sliding_window_b200(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window_size: int | None,
                        dropout_p: float) -> bool:
    """Whether a call on [B, T, H, D] q, k, v takes the tcgen05 path for its sliding
    window: SDPA has no sliding-window kernel (a mask makes it run every key; measured
    at [16, 2048, 6, 128], window 512: forward 363 us vs 109 us, forward + backward
    1.58 ms vs 0.73 ms), so every backend name but ``"torch"`` sends a window shorter
    than the sequence here when the shapes allow it."""
    return (window_size is not None and 0 < window_size < q.shape[1] and not dropout_p
            and (q.is_cuda or q.is_meta) and ops.attention_supported(q, k, v))


def attention_b200(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, window_size: int | None) -> torch.Tensor:
    """Causal attention on [B, T, H, 128] bf16 q, k, v (the QKV kernel's layout, no
    transposes): the tcgen05 forward of hlm_attention_fwd; gradients through the tcgen05
    backward (hlm_attention_bwd) for a sliding window and cuDNN's SDPA backward for full
    causal attention (ops.attention_backward).
    ``window_size`` keys per query (the FlashAttention window ``(window_size - 1, 0)``,
    kernels.py:839) or None for full causal."""
    _cuda_only(q, "attention_b200")
    if not ops.attention_supported(q, k, v):
        raise RuntimeError("attention_b200: needs [B, T, H, 128] bf16 q, k, v with T a multiple of 128")
    out, _ = ops.attention(q, k, v, 0 if window_size is None else int(window_size), 1.0 / math.sqrt(q.shape[-1]))
    return out


def scaled_dot_product_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, dropout_p: float,
                                 is_causal: bool = True, attn_mask: torch.Tensor | None = None,
                                 block_mask: Any | None = None, window_size: int | None = None,
                                 backend: str = "flash_attn_2") -> torch.Tensor:
    """Attention core with the reference's signature and backend names (kernels.py:774-847).

    Layouts follow the reference: ``"torch"``, ``"sdpa"`` and
    ``"flex_attention"`` take and return [B, H, T, D]; the FlashAttention
    names take and return [B, T, H, D] (the reference's ``fwd_flash_attn_*``
    pass q, k, v without transposing, model.py:213-251).  Every name except
    ``"torch"`` runs torch SDPA (the attention core named by the benchmark
    configuration) for full causal attention and this library's tcgen05 forward
    for a sliding window where the shapes allow it (``sliding_window_b200``), so the
    reference's ``AttentionCore`` runs unmodified on this module.  ``"torch"`` is the reference's explicit softmax
    (kernels.py:785-800).  The argument checks are the reference's: the
    FlashAttention names reject an explicit mask and (but for flash_attn_2)
    dropout, flex_attention rejects dropout.
    """
    if backend == "sdpa":
        if attn_mask is None and is_causal:
            qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
            if sliding_window_b200(qt, kt, vt, window_size, dropout_p):
                return attention_b200(qt, kt, vt, window_size).transpose(1, 2)
        return _sdpa_core(q, k, v, dropout_p, is_causal, attn_mask, window_size)
    if backend in _FLASH_BACKENDS:
        if attn_mask is not None:
            raise RuntimeError(f"{backend} path expects window_size instead of an explicit attention mask")
        if dropout_p and backend != "flash_attn_2":
            raise RuntimeError(f"{backend} backend does not support dropout")
        if is_causal and sliding_window_b200(q, k, v, window_size, dropout_p):
            return attention_b200(q, k, v, window_size)
        q, k, v = (t.bfloat16().transpose(1, 2) for t in (q, k, v))
        return _sdpa_core(q, k, v, dropout_p, is_causal, None, window_size).transpose(1, 2)
    if backend == "flex_attention":
        if dropout_p:
            raise RuntimeError("flex_attention backend does not support dropout")
        if block_mask is not None:
            if not isinstance(block_mask, WindowBlockMask):
                raise RuntimeError("flex_attention on this path takes the mask made by "
                                   "flex_attention_block_mask (causal, optional sliding window)")
            if block_mask.seq_len != q.shape[-2]:
                raise RuntimeError(f"block mask is for seq_len {block_mask.seq_len}, got {q.shape[-2]}")
            window_size = block_mask.window_size
        qt, kt, vt = (t.transpose(1, 2) for t in (q, k, v))
        if sliding_window_b200(qt, kt, vt, window_size, 0.0):
            return attention_b200(qt, kt, vt, window_size).transpose(1, 2)
        return _sdpa_core(q, k, v, 0.0, True, None, window_size)
    if backend == "torch":
        if window_size is not None and attn_mask is None:
            # the reference's caller passes its window as attn_mask (model.py:185-194);
            # a caller that passes only window_size gets the same mask
            pos = torch.arange(q.shape[-2], device=q.device)
            dist = pos[:, None] - pos[None, :]
            attn_mask = (dist >= 0) & (dist < window_size)
        scale = 1.0 / math.sqrt(q.shape[-1])
        attn = torch.matmul(q, k.transpose(-2, -1)) * scale
        if is_causal:
            q_len, kv_len = q.shape[-2], k.shape[-2]
            causal = torch.ones((q_len, kv_len), device=q.device, dtype=torch.bool).tril()
            attn = attn.masked_fill(~causal, float("-inf"))
        if attn_mask is not None:
            if attn_mask.dtype == torch.bool:
                attn = attn.masked_fill(~attn_mask, float("-inf"))
            else:
                attn = attn + attn_mask
        attn = torch.softmax(attn.float(), dim=-1).to(dtype=q.dtype)
        if dropout_p:
            attn = F.dropout(attn, p=dropout_p, training=True)
        return torch.matmul(attn, v)
    raise RuntimeError(f"unsupported attention backend {backend!r}")


def apply_precision_policy(model: torch.nn.Module, precision: str,
                           allow_torch_backend: bool = False) -> torch.nn.Module:
    """Cast floating parameters (and grads) to bf16 (kernels.py:962-972)."""
    if precision == "bf16":
        for param in model.parameters():
            if param.is_floating_point():
                param.data = param.data.to(dtype=torch.bfloat16)
                if param.grad is not None:
                    param.grad.data = param.grad.data.to(dtype=torch.bfloat16)
        return model
    if precision in {"fp32_test", "bf16_test"} and allow_torch_backend:
        return model
    raise RuntimeError(f"unsupported precision mode {precision!r}; the training fast path uses bf16")
