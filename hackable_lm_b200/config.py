"""Model/backends configuration used by the B200 path.

Restates the parts of the reference ``config.py`` that the operator layer and
the data-parallel training step read: backend names and fields
(config.py:10-18), the depth-scaled model dimensions (config.py:80-83,
145-147, 150-162), the per-layer attention window (config.py:184-191) and
the FLOPs-per-token estimate (config.py:194-207).  The reference's
budget/learning-rate scheduling machinery is not part of this path.
"""
from __future__ import annotations

from dataclasses import asdict, dataclass, field
from typing import Any

# "triton" is kept as an accepted value so that reference configs select the
# B200 kernels unchanged; it resolves to "b200".
MODULE_BACKENDS = {"torch", "triton", "b200"}
# "sdpa" is this path's attention core (torch SDPA); "b200" the tcgen05 forward
# (hlm_attention_fwd) with the tcgen05 backward for sliding windows and cuDNN's
# for full causal attention; the reference's names (config.py:11) are accepted too
# and run on SDPA (sliding-window layers on the tcgen05 kernels), so reference
# configs and their default "flash_attn_2" select it unchanged.
ATTENTION_BACKENDS = {"torch", "sdpa", "b200", "flex_attention", "flash_attn_2", "flash_attn_3", "flash_attn_4"}
MODULE_BACKEND_FIELDS = (
    "qkv_backend",
    "output_backend",
    "gate_up_backend",
    "down_backend",
    "lm_head_backend",
)

DEFAULTS = {
    "head_dim": 128,
    "layers_per_head": 2,
    "sequence_len": 2048,
    "device_batch_size": 16,
    "global_batch_tokens": 2**20,
    "attention_window": 512,
    "attention_full_every": 4,
    "loss_chunk_size": 4096,
}


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


def normalize_module_backend(name: str, backend: str) -> str:
    if not isinstance(backend, str) or backend.lower() not in MODULE_BACKENDS:
        raise ValueError(f"unknown {name} {backend!r}")
    backend = backend.lower()
    return "b200" if backend == "triton" else backend


def normalize_attention_backend(backend: str) -> str:
    if not isinstance(backend, str) or backend.lower() not in ATTENTION_BACKENDS:
        raise ValueError(f"unknown attention_backend {backend!r}")
    return backend.lower()


def depth_dimensions(depth: int, head_dim: int = DEFAULTS["head_dim"],
                     layers_per_head: int = DEFAULTS["layers_per_head"]) -> tuple[int, int]:
    n_head = ceil_div(depth, layers_per_head)
    return n_head * head_dim, n_head


def mlp_hidden_dim(n_embd: int) -> int:
    hidden = ceil_div(8 * n_embd, 3)
    return ceil_div(hidden, 256) * 256


def scaling_params_for_depth(depth: int, vocab_size: int) -> int:
    n_embd, _ = depth_dimensions(depth)
    hidden = mlp_hidden_dim(n_embd)
    return depth * (4 * n_embd * n_embd + 3 * n_embd * hidden) + n_embd * vocab_size


def layer_attention_window(layer_idx: int, n_layer: int, attention_window: int | None,
                           attention_full_every: int | None) -> int | None:
    if attention_window is None:
        return None
    if layer_idx == n_layer - 1:
        return None
    if attention_full_every is not None and (layer_idx + 1) % attention_full_every == 0:
        return None
    return attention_window


def estimate_flops_per_token(depth: int, n_embd: int, seq_len: int, scaling_params: int,
                             attention_window: int | None = None,
                             attention_full_every: int | None = None) -> int:
    attn = 0
    for layer_idx in range(depth):
        w = layer_attention_window(layer_idx, depth, attention_window, attention_full_every)
        ctx = seq_len if w is None else min(seq_len, w)
        attn += 12 * ctx * n_embd
    return int(6 * scaling_params + attn)


@dataclass
class ModelConfig:
    """Decoder-only model: RoPE, pre-norm RMSNorm, QK norm, SwiGLU MLP (config.py:210-234)."""

    vocab_size: int
    block_size: int
    n_layer: int
    n_embd: int
    n_head: int
    n_kv_head: int
    head_dim: int = DEFAULTS["head_dim"]
    mlp_hidden: int = 0
    rope_theta: float = 1_000_000.0
    rope_fraction: float = 0.25
    norm_eps: float = 1e-6
    dropout: float = 0.0
    attention_window: int | None = None
    attention_full_every: int | None = DEFAULTS["attention_full_every"]
    attention_backend: str = "sdpa"
    loss_chunk_size: int | None = DEFAULTS["loss_chunk_size"]
    qkv_backend: str = "b200"
    output_backend: str = "b200"
    gate_up_backend: str = "b200"
    down_backend: str = "b200"
    lm_head_backend: str = "b200"
    extra: dict[str, Any] = field(default_factory=dict)

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)


def model_config_for_depth(depth: int, *, vocab_size: int = 32768, sequence_len: int = 2048,
                           attention_window: int | None = None, backend: str = "b200",
                           attention_backend: str = "sdpa", **overrides: Any) -> ModelConfig:
    """ModelConfig as resolve_config builds it (config.py:433-446)."""
    n_embd, n_head = depth_dimensions(depth)
    backends = {name: normalize_module_backend(name, overrides.pop(name, backend))
                for name in MODULE_BACKEND_FIELDS}
    return ModelConfig(
        vocab_size=vocab_size,
        block_size=sequence_len,
        n_layer=depth,
        n_embd=n_embd,
        n_head=n_head,
        n_kv_head=n_head,
        mlp_hidden=mlp_hidden_dim(n_embd),
        attention_window=attention_window,
        attention_backend=normalize_attention_backend(attention_backend),
        **backends,
        **overrides,
    )


def gradient_accumulation(global_batch_tokens: int, device_batch_size: int, sequence_len: int,
                          world_size: int) -> int:
    """Per-rank micro-steps that keep the global batch (config.py:420-422, train.py:872-886)."""
    micro = device_batch_size * sequence_len
    total = max(1, ceil_div(global_batch_tokens, micro))
    if world_size > 1:
        if total <= 1:
            raise RuntimeError("DDP is only enabled when gradient_accumulation_steps > 1.")
        if total % world_size != 0:
            raise RuntimeError(
                "DDP requires gradient_accumulation_steps to divide evenly by WORLD_SIZE "
                f"to preserve global_batch_tokens: got gradient_accumulation_steps={total}, "
                f"WORLD_SIZE={world_size}."
            )
    return total // max(1, world_size)
