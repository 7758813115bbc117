"""Decoder-only language model whose hot-path modules run the B200 operators.

Module and parameter names follow the reference ``model.py`` one to one
(``tok_emb``, ``blocks.N.attn.qkv.qkv_proj``, ``blocks.N.attn.out.o_proj``,
``blocks.N.mlp.gate_up.gate_up_proj``, ``blocks.N.mlp.down.down_proj``,
``lm_head.lm_head``), so reference state dicts load unchanged.  Every
``AcceleratedModule`` dispatches ``fwd_<backend>`` from its config field
(model.py:19-38): ``"torch"`` is the reference's own formulation (used on the
CPU), ``"b200"`` the hand-written sm_100a kernels:

* QKVProjection.fwd_b200     -> fused tcgen05 GEMM + QK-norm + RoPE (qkv_rope)
* OutputProjection.fwd_b200  -> o_proj GEMM with the residual add + RMSNorm in
  its epilogue (one cluster of CTAs per 128-row block exchanges row sums)
* GateUpProjection.fwd_b200  -> gate_up GEMM with the SwiGLU in its epilogue
* DownProjection.fwd_b200    -> down GEMM with the residual add + RMSNorm in its epilogue
* MLP (both of the above on b200) -> gate_up_swiglu + swiglu_down_residual_norm:
  the down GEMM's backward computes grad_h and the SwiGLU backward in one kernel
* LMHeadProjection.fwd_b200  -> fused LM head + cross-entropy
* input norm                 -> RMSNorm kernel

The attention core is torch SDPA (flash kernels on B200), causal.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch import nn

from . import kernels, ops
from .config import ModelConfig, layer_attention_window


def rms_norm_torch(x: torch.Tensor, weight: torch.Tensor | None, eps: float) -> torch.Tensor:
    """Reference formulation (model.py:14-16)."""
    y = x * torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
    return y if weight is None else y * weight


def residual_rms_norm_torch(residual: torch.Tensor, branch: torch.Tensor, eps: float):
    """Reference formulation (model.py:73-75)."""
    out = residual + branch
    return out, rms_norm_torch(out, None, eps)


class AcceleratedModule(nn.Module):
    backend_attr: str | None = None

    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config

    def selected_backend(self) -> str:
        if self.backend_attr is None:
            return "torch"
        backend = getattr(self.config, self.backend_attr)
        return "b200" if backend == "triton" else backend

    def forward(self, *args, **kwargs):
        backend = self.selected_backend()
        fn = getattr(self, f"fwd_{backend}", None)
        if fn is None:
            raise RuntimeError(f"{type(self).__name__} does not support backend {backend!r}")
        return fn(*args, **kwargs)


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6, param: bool = False, backend: str = "torch") -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim)) if param else None
        self.backend = backend

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.backend == "b200" and (x.is_cuda or x.is_meta):
            return kernels.rms_norm(x, self.weight, self.eps)
        return rms_norm_torch(x, self.weight, self.eps)


class RotaryEmbedding(nn.Module):
    """cos/sin cache [1, 1, T, rotary_dim] (model.py:50-70)."""

    def __init__(self, dim: int, theta: float = 1_000_000.0, fraction: float = 0.25) -> None:
        super().__init__()
        rotary_dim = int(dim * fraction)
        rotary_dim -= rotary_dim % 2
        self.rotary_dim = rotary_dim
        inv_freq = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2).float() / rotary_dim))
        self.register_buffer("inv_freq", inv_freq, persistent=False)
        self._cache: dict = {}

    def forward(self, seq_len: int, device: torch.device, dtype: torch.dtype):
        key = (seq_len, str(device), dtype)
        if key not in self._cache:
            t = torch.arange(seq_len, device=device, dtype=self.inv_freq.dtype)
            freqs = torch.outer(t, self.inv_freq.to(device))
            emb = torch.cat((freqs, freqs), dim=-1)
            self._cache[key] = (emb.cos()[None, None].to(dtype), emb.sin()[None, None].to(dtype))
        return self._cache[key]


class QKVProjection(AcceleratedModule):
    backend_attr = "qkv_backend"

    def __init__(self, config: ModelConfig, layer_idx: int) -> None:
        super().__init__(config)
        self.n_head = config.n_head
        self.n_kv_head = config.n_kv_head
        self.head_dim = config.head_dim
        self.q_dim = config.n_head * config.head_dim
        self.kv_dim = config.n_kv_head * config.head_dim
        self.qkv_proj = nn.Linear(config.n_embd, self.q_dim + 2 * self.kv_dim, bias=False)
        self.rope = RotaryEmbedding(config.head_dim, config.rope_theta, config.rope_fraction)

    def fwd_torch(self, x: torch.Tensor):
        """model.py:92-115."""
        bsz, seq_len, _ = x.shape
        q, k, v = self.qkv_proj(x).split((self.q_dim, self.kv_dim, self.kv_dim), dim=-1)
        q = q.view(bsz, seq_len, self.n_head, self.head_dim)
        k = k.view(bsz, seq_len, self.n_kv_head, self.head_dim)
        v = v.view(bsz, seq_len, self.n_kv_head, self.head_dim)
        cos, sin = self.rope(seq_len, x.device, q.dtype)
        cos, sin = cos.transpose(1, 2), sin.transpose(1, 2)
        half = cos.shape[-1] // 2
        rd = cos.shape[-1]

        def rope(t):
            t = rms_norm_torch(t, None, self.config.norm_eps)
            t1, t2, tp = t[..., :half], t[..., half:rd], t[..., rd:]
            c, s = cos[..., :half], sin[..., :half]
            return torch.cat((t1 * c - t2 * s, t2 * c + t1 * s, tp), dim=-1)

        return rope(q), rope(k), v

    def fwd_b200(self, x: torch.Tensor):
        cos, sin = self.rope(x.shape[1], x.device, x.dtype)
        return kernels.qkv_projection_rope(x, self.qkv_proj.weight, cos, sin, self.n_head, self.n_kv_head,
                                           self.config.norm_eps)


class AttentionCore(nn.Module):
    def __init__(self, config: ModelConfig, layer_idx: int) -> None:
        super().__init__()
        self.config = config
        self.n_head = config.n_head
        self.n_kv_head = config.n_kv_head
        self.window = layer_attention_window(layer_idx, config.n_layer, config.attention_window,
                                             config.attention_full_every)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        seq_len = q.shape[1]
        window = self.window if self.window is not None and self.window < seq_len else None
        backend = self.config.attention_backend
        if backend != "torch" and self.config.dropout == 0.0 and (
                (backend == "b200" and (q.is_cuda or q.is_meta) and ops.attention_supported(q, k, v))
                or kernels.sliding_window_b200(q, k, v, window, 0.0)):
            # tcgen05 forward on the [B, T, H, D] layout the QKV kernel wrote: every
            # layer with "b200", and the sliding-window layers with every other name
            # (SDPA has no sliding-window kernel)
            return kernels.attention_b200(q, k, v, window)
        q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if self.n_kv_head != self.n_head:
            rep = self.n_head // self.n_kv_head
            k = k.repeat_interleave(rep, dim=1)
            v = v.repeat_interleave(rep, dim=1)
        backend = "torch" if q.device.type == "cpu" else backend
        y = kernels.scaled_dot_product_attention(q, k, v, 0.0, is_causal=True, window_size=window,
                                                 backend=backend)
        return y.transpose(1, 2)


class OutputProjection(AcceleratedModule):
    backend_attr = "output_backend"

    def __init__(self, config: ModelConfig) -> None:
        super().__init__(config)
        self.norm_eps = config.norm_eps
        self.o_proj = nn.Linear(config.n_head * config.head_dim, config.n_embd, bias=False)

    def fwd_torch(self, y: torch.Tensor, residual: torch.Tensor):
        b, t, h, d = y.shape
        return residual_rms_norm_torch(residual, self.o_proj(y.reshape(b, t, h * d)), self.norm_eps)

    def fwd_b200(self, y: torch.Tensor, residual: torch.Tensor):
        b, t, h, d = y.shape
        y2 = y.reshape(b, t, h * d)
        w = self.o_proj.weight
        if ops.proj_norm_supported(y2, w) and residual.dtype == y2.dtype:
            # o_proj GEMM with the residual add and RMSNorm in its epilogue
            return ops.proj_residual_norm(y2, w, residual, self.norm_eps)
        return kernels.residual_rms_norm(residual, self.o_proj(y2), self.norm_eps)


class CausalSelfAttention(nn.Module):
    def __init__(self, config: ModelConfig, layer_idx: int) -> None:
        super().__init__()
        self.qkv = QKVProjection(config, layer_idx)
        self.attention = AttentionCore(config, layer_idx)
        self.out = OutputProjection(config)

    def forward(self, x: torch.Tensor, residual: torch.Tensor):
        q, k, v = self.qkv(x)
        return self.out(self.attention(q, k, v), residual)


class GateUpProjection(AcceleratedModule):
    backend_attr = "gate_up_backend"

    def __init__(self, config: ModelConfig) -> None:
        super().__init__(config)
        self.gate_up_proj = nn.Linear(config.n_embd, 2 * config.mlp_hidden, bias=False)

    def fwd_torch(self, x: torch.Tensor) -> torch.Tensor:
        gate, up = self.gate_up_proj(x).chunk(2, dim=-1)
        return F.silu(gate) * up

    def fwd_b200(self, x: torch.Tensor) -> torch.Tensor:
        w = self.gate_up_proj.weight
        if ops.gate_up_swiglu_supported(x, w):
            # the GEMM with the SwiGLU activation in its epilogue
            return ops.gate_up_swiglu(x, w)[0]
        return kernels.swiglu_triton(self.gate_up_proj(x))


class DownProjection(AcceleratedModule):
    backend_attr = "down_backend"

    def __init__(self, config: ModelConfig) -> None:
        super().__init__(config)
        self.norm_eps = config.norm_eps
        self.down_proj = nn.Linear(config.mlp_hidden, config.n_embd, bias=False)

    def fwd_torch(self, x: torch.Tensor, residual: torch.Tensor):
        return residual_rms_norm_torch(residual, self.down_proj(x), self.norm_eps)

    def fwd_b200(self, x: torch.Tensor, residual: torch.Tensor):
        w = self.down_proj.weight
        if ops.proj_norm_supported(x, w) and residual.dtype == x.dtype:
            return ops.proj_residual_norm(x, w, residual, self.norm_eps)
        return kernels.residual_rms_norm(residual, self.down_proj(x), self.norm_eps)


class MLP(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.gate_up = GateUpProjection(config)
        self.down = DownProjection(config)

    def forward(self, x: torch.Tensor, residual: torch.Tensor):
        if self.gate_up.selected_backend() == "b200" and self.down.selected_backend() == "b200":
            w_gu = self.gate_up.gate_up_proj.weight
            w_dn = self.down.down_proj.weight
            if ops.gate_up_swiglu_supported(x, w_gu) and ops.swiglu_down_supported(w_gu, w_dn):
                # gate_up GEMM with the SwiGLU in its epilogue, then the down GEMM (residual
                # add + RMSNorm in its epilogue) whose backward computes grad_h and the
                # SwiGLU backward in one kernel
                h, gate_up = ops.gate_up_swiglu(x, w_gu)
                if ops.proj_norm_supported(h, w_dn) and residual.dtype == h.dtype:
                    return ops.swiglu_down_residual_norm(h, gate_up, w_dn, residual, self.down.norm_eps)
                y = ops.swiglu_down(h, gate_up, w_dn)
                return kernels.residual_rms_norm(residual, y, self.down.norm_eps)
        return self.down(self.gate_up(x), residual)


class LMHeadProjection(AcceleratedModule):
    backend_attr = "lm_head_backend"

    def __init__(self, config: ModelConfig) -> None:
        super().__init__(config)
        self.lm_head = nn.Linear(config.n_embd, config.vocab_size, bias=False)
        self.chunk_size = config.loss_chunk_size

    def fwd_torch(self, hidden: torch.Tensor, targets: torch.Tensor | None = None):
        """model.py:325-339 (mean over all tokens, default ignore_index)."""
        if targets is None:
            return self.lm_head(hidden), None
        h = hidden.reshape(-1, hidden.size(-1))
        t = targets.reshape(-1)
        n = t.numel()
        chunk = self.chunk_size or n
        loss_sum = h.new_zeros((), dtype=torch.float32)
        for s in range(0, n, chunk):
            e = min(s + chunk, n)
            logits = F.linear(h[s:e], self.lm_head.weight)
            loss_sum = loss_sum + F.cross_entropy(logits.float(), t[s:e], reduction="sum")
        return None, loss_sum / n

    def fwd_b200(self, hidden: torch.Tensor, targets: torch.Tensor | None = None):
        if targets is None:
            return self.lm_head(hidden), None
        loss = kernels.fused_linear_cross_entropy_with_weight(hidden, self.lm_head.weight, None, targets,
                                                              backend="b200", chunk_size=self.chunk_size)
        return None, loss


class Block(nn.Module):
    def __init__(self, config: ModelConfig, layer_idx: int) -> None:
        super().__init__()
        self.attn = CausalSelfAttention(config, layer_idx)
        self.mlp = MLP(config)

    def forward(self, x: torch.Tensor, x_norm: torch.Tensor):
        x, x_norm = self.attn(x_norm, x)
        x, x_norm = self.mlp(x_norm, x)
        return x, x_norm


class LanguageModel(nn.Module):
    def __init__(self, config: ModelConfig) -> None:
        super().__init__()
        self.config = config
        self.tok_emb = nn.Embedding(config.vocab_size, config.n_embd)
        norm_backend = "b200" if config.output_backend in ("b200", "triton") else "torch"
        self.input_norm = RMSNorm(config.n_embd, config.norm_eps, backend=norm_backend)
        self.blocks = nn.ModuleList([Block(config, i) for i in range(config.n_layer)])
        self.lm_head = LMHeadProjection(config)
        self.apply(self._init_weights)
        for name, param in self.named_parameters():
            if name.endswith("o_proj.weight") or name.endswith("down_proj.weight"):
                nn.init.normal_(param, mean=0.0, std=0.02 / math.sqrt(2 * config.n_layer))

    @staticmethod
    def _init_weights(module: nn.Module) -> None:
        """GPT-style init (model.py:376-380)."""
        if isinstance(module, (nn.Linear, nn.Embedding)):
            nn.init.normal_(module.weight, mean=0.0, std=0.02)

    def forward(self, idx: torch.Tensor, targets: torch.Tensor | None = None):
        x = self.tok_emb(idx)
        x_norm = self.input_norm(x)
        for block in self.blocks:
            x, x_norm = block(x, x_norm)
        return self.lm_head(x_norm, targets)

    def parameter_count(self) -> int:
        return sum(p.numel() for p in self.parameters())
