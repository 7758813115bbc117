"""Data-parallel training step of the depth-12 decoder on the B200 operators.

Mirrors the reference training loop's per-step work (train.py:67-89,
872-886, 926-1018): one process per GPU (torchrun env), the model cast to
bf16 (bf16 parameters and gradients), DistributedDataParallel with 25 MB
bf16 gradient buckets over NCCL, gradient accumulation with ``no_sync`` on all
but the last micro-step so the global batch is preserved
(grad_accum = global_tokens / (micro_batch * seq_len * world)), then the
Muon/AdamW optimizer step (Muon's Newton-Schulz work sharded across the ranks,
then one all-gather of the updated matrices).  Data is synthetic (uniform token
ids; targets are the ids shifted by one), so the data loader is not part of
the step.
"""
from __future__ import annotations

import contextlib
import os
from dataclasses import dataclass

import torch

from . import kernels
from .config import DEFAULTS, ModelConfig, gradient_accumulation, model_config_for_depth
from .model import LanguageModel
from .optim import MuonAdamW

D12 = {"depth": 12, "vocab": 32768, "seq_len": 2048, "micro_batch": 16, "global_tokens": 2**20}


@dataclass
class StepSetup:
    model: torch.nn.Module        # the bf16 LanguageModel
    train_model: torch.nn.Module  # DDP wrapper (or the model itself on one GPU)
    optimizer: MuonAdamW
    config: ModelConfig
    accum: int
    world: int
    micro_batch: int
    seq_len: int


def lr_settings(depth: int) -> dict:
    """Learning rates as resolve_config derives them (config.py:424-431)."""
    import math

    scale = min(1.0, math.sqrt(6 / depth))
    return {"embedding_lr": 0.1 * scale, "unembedding_lr": 0.01 * scale, "matrix_lr": 0.02 * scale,
            "scalar_lr": 0.1 * scale, "weight_decay": 0.1}


def build(device: torch.device, *, depth: int = D12["depth"], vocab: int = D12["vocab"],
          seq_len: int = D12["seq_len"], micro_batch: int = D12["micro_batch"],
          global_tokens: int = D12["global_tokens"], world: int = 1, backend: str = "b200",
          attention_window: int | None = None, seed: int = 0, ddp: bool | None = None) -> StepSetup:
    torch.manual_seed(seed)
    cfg = model_config_for_depth(depth, vocab_size=vocab, sequence_len=seq_len,
                                 attention_window=attention_window, backend=backend,
                                 attention_backend="sdpa" if device.type == "cuda" else "torch")
    model = LanguageModel(cfg).to(device)
    kernels.apply_precision_policy(model, "bf16")
    opt = MuonAdamW(model, n_head=cfg.n_head, n_kv_head=cfg.n_kv_head, head_dim=cfg.head_dim,
                    **lr_settings(depth))
    accum = gradient_accumulation(global_tokens, micro_batch, seq_len, world)
    use_ddp = (world > 1) if ddp is None else ddp
    train_model = model
    if use_ddp:
        from torch.nn.parallel import DistributedDataParallel

        kw = {"device_ids": [device.index]} if device.type == "cuda" else {}
        train_model = DistributedDataParallel(model, bucket_cap_mb=25, gradient_as_bucket_view=True, **kw)
    return StepSetup(model, train_model, opt, cfg, accum, world, micro_batch, seq_len)


def synthetic_batches(n: int, micro_batch: int, seq_len: int, vocab: int, rank: int, device,
                      seed: int = 1234) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """n distinct micro-batches of uniform token ids; targets = ids shifted by one."""
    g = torch.Generator().manual_seed(seed + 7919 * rank)
    out = []
    for _ in range(n):
        ids = torch.randint(0, vocab, (micro_batch, seq_len + 1), generator=g)
        out.append((ids[:, :-1].contiguous().to(device), ids[:, 1:].contiguous().to(device)))
    return out


def train_step(s: StepSetup, batches, fetch=None, optimizer_step: bool = True, max_grad_norm: float = 0.0,
               mark=None) -> torch.Tensor:
    """One optimizer step over s.accum micro-batches; returns the mean loss (device tensor).

    ``fetch(i)`` may supply micro-batch i (e.g. copied from host memory);
    otherwise batches are cycled from the resident list.  With
    ``optimizer_step=False`` the averaged gradients are left in ``.grad``.
    ``max_grad_norm > 0`` clips the global gradient norm before the optimizer
    step, as the reference's ``--max-grad-norm`` does (train.py:1004-1005; its
    default, 0, skips it).  ``mark(tag)``, when given, is called after each
    micro-step ("micro"), after clipping ("clip") and after the optimizer step
    ("opt"), so a caller can record CUDA events for a per-phase breakdown.
    """
    s.optimizer.zero_grad()
    total = None
    ddp = s.train_model is not s.model
    for i in range(s.accum):
        x, y = fetch(i) if fetch is not None else batches[i % len(batches)]
        ctx = s.train_model.no_sync() if (ddp and i < s.accum - 1) else contextlib.nullcontext()
        with ctx:
            _, loss = s.train_model(x, y)
            (loss / s.accum).backward()
        total = loss.detach() if total is None else total + loss.detach()
        if mark is not None:
            mark("micro")
    if max_grad_norm > 0:
        torch.nn.utils.clip_grad_norm_(s.optimizer.parameters(), max_grad_norm, foreach=True)
    if mark is not None:
        mark("clip")
    if optimizer_step:
        s.optimizer.step()
    if mark is not None:
        mark("opt")
    return total / s.accum


def world_from_env() -> tuple[int, int, int]:
    return (int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0")),
            int(os.environ.get("LOCAL_RANK", "0")))


__all__ = ["D12", "DEFAULTS", "StepSetup", "build", "synthetic_batches", "train_step", "world_from_env"]
