"""CPU restatement of the reference decoder forward/backward (test infrastructure only).

Functional form of the reference LanguageModel (model.py:355-391) with the
torch backends: embedding, weightless input RMSNorm, per layer QKV projection
+ QK-norm + RoPE (model.py:101-115), causal softmax attention in the
reference's explicit formulation (kernels.py:785-800), o_proj + residual-add +
RMSNorm, gate_up + SwiGLU, down + residual-add + RMSNorm, and the chunked
LM-head cross-entropy (model.py:325-339).  Used by bench.py for the CPU
baseline of the training step.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .hotpath import apply_partial_rope, rms_norm, rope_tables


def init_params(vocab=32768, n_layer=12, n_embd=768, n_head=6, head_dim=128, mlp_hidden=2048, seed=0,
                dtype=torch.float32):
    """GPT-style init as the reference (model.py:368-380)."""
    g = torch.Generator().manual_seed(seed)

    def normal(*shape, std):
        return (torch.randn(*shape, generator=g) * std).to(dtype)

    proj_std = 0.02 / math.sqrt(2 * n_layer)
    p = {"tok_emb": normal(vocab, n_embd, std=0.02), "lm_head": normal(vocab, n_embd, std=0.02)}
    for i in range(n_layer):
        p[f"{i}.qkv"] = normal(3 * n_head * head_dim, n_embd, std=0.02)
        p[f"{i}.o"] = normal(n_embd, n_head * head_dim, std=proj_std)
        p[f"{i}.gate_up"] = normal(2 * mlp_hidden, n_embd, std=0.02)
        p[f"{i}.down"] = normal(n_embd, mlp_hidden, std=proj_std)
    return p


def forward_loss(p, idx, targets, n_layer=12, n_head=6, head_dim=128, eps=1e-6, rope_theta=1_000_000.0,
                 rope_fraction=0.25, loss_chunk=4096):
    B, T = idx.shape
    cos, sin = rope_tables(head_dim, T, rope_theta, rope_fraction)
    cos, sin = cos.transpose(1, 2), sin.transpose(1, 2)
    x = p["tok_emb"][idx]
    x_norm = rms_norm(x, None, eps)
    causal = torch.ones(T, T, dtype=torch.bool).tril()
    for i in range(n_layer):
        qkv = x_norm @ p[f"{i}.qkv"].t()
        q, k, v = qkv.split((n_head * head_dim,) * 3, dim=-1)
        q = apply_partial_rope(rms_norm(q.reshape(B, T, n_head, head_dim), None, eps), cos, sin)
        k = apply_partial_rope(rms_norm(k.reshape(B, T, n_head, head_dim), None, eps), cos, sin)
        v = v.reshape(B, T, n_head, head_dim)
        qh, kh, vh = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        att = (qh @ kh.transpose(-2, -1)) / math.sqrt(head_dim)
        att = att.masked_fill(~causal, float("-inf")).softmax(dim=-1)
        y = (att @ vh).transpose(1, 2).reshape(B, T, n_head * head_dim)
        x = x + y @ p[f"{i}.o"].t()
        x_norm = rms_norm(x, None, eps)
        gate, up = (x_norm @ p[f"{i}.gate_up"].t()).chunk(2, dim=-1)
        x = x + (F.silu(gate) * up) @ p[f"{i}.down"].t()
        x_norm = rms_norm(x, None, eps)
    h = x_norm.reshape(-1, x_norm.shape[-1])
    t = targets.reshape(-1)
    loss = h.new_zeros(())
    for s in range(0, h.shape[0], loss_chunk):
        logits = h[s:s + loss_chunk] @ p["lm_head"].t()
        loss = loss + F.cross_entropy(logits, t[s:s + loss_chunk], reduction="sum")
    return loss / t.numel()


def train_step_cpu(p, idx, targets, **kw):
    """One forward + backward (autograd) of the restated model; returns the loss."""
    leaves = {k: v.detach().requires_grad_(True) for k, v in p.items()}
    loss = forward_loss(leaves, idx, targets, **kw)
    loss.backward()
    return float(loss.detach())
