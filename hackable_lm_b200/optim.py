"""Muon + AdamW optimizer step for the data-parallel training step.

The optimizer is outside the operator hot path; this is a compact eager
PyTorch restatement of the reference's MuonAdamW (optim.py:20-75, 313-329,
403-452) so that the training step includes the same per-step work:

* AdamW (betas 0.9/0.95, eps 1e-8, bf16 moments) for the embedding and the
  LM head (optim.py:20-43);
* Muon for the 2-D block matrices, stacked by shape, with qkv_proj split into
  its q/k/v row blocks and gate_up_proj into gate/up halves (optim.py:387-399):
  bf16 momentum lerp, Nesterov-style blend, Frobenius normalisation, five
  Newton-Schulz iterations with coefficients (3.4445, -4.7750, 2.0315), then
  decoupled weight decay and the update (optim.py:46-75).
"""
from __future__ import annotations

from typing import Any

import torch

MUON_NAME_MARKERS = ("qkv_proj.weight", "o_proj.weight", "gate_up_proj.weight", "down_proj.weight")
NS_COEFFS = (3.4445, -4.7750, 2.0315)


def _muon_split_sizes(name: str, param: torch.Tensor, n_head: int, n_kv_head: int, head_dim: int):
    if name.endswith("qkv_proj.weight"):
        return (n_head * head_dim, n_kv_head * head_dim, n_kv_head * head_dim)
    if name.endswith("gate_up_proj.weight"):
        return (param.shape[0] // 2, param.shape[0] // 2)
    return None


@torch.no_grad()
def newton_schulz5(x: torch.Tensor) -> torch.Tensor:
    """Batched quintic Newton-Schulz orthogonalisation in bf16 (optim.py:58-68)."""
    a, b, c = NS_COEFFS
    x = x.bfloat16()
    x = x / (x.norm(dim=(-2, -1), keepdim=True) + 1e-7)
    if x.size(-2) > x.size(-1):
        for _ in range(5):
            xtx = x.mT @ x
            poly = torch.baddbmm(xtx, xtx, xtx, beta=b, alpha=c)
            x = torch.baddbmm(x, x, poly, beta=a)
    else:
        for _ in range(5):
            xxt = x @ x.mT
            poly = torch.baddbmm(xxt, xxt, xxt, beta=b, alpha=c)
            x = torch.baddbmm(x, poly, x, beta=a)
    return x


class MuonAdamW:
    def __init__(self, model: torch.nn.Module, *, embedding_lr: float, unembedding_lr: float,
                 matrix_lr: float, scalar_lr: float, weight_decay: float, n_head: int, n_kv_head: int,
                 head_dim: int) -> None:
        self.adamw: list[dict[str, Any]] = []
        muon: dict[tuple, list[torch.nn.Parameter]] = {}
        emb, unemb, scalar = [], [], []
        for name, p in model.named_parameters():
            if not p.requires_grad:
                continue
            if p.ndim == 2 and any(m in name for m in MUON_NAME_MARKERS):
                split = _muon_split_sizes(name, p, n_head, n_kv_head, head_dim)
                muon.setdefault((tuple(p.shape), split), []).append(p)
            elif "tok_emb" in name:
                emb.append(p)
            elif "lm_head" in name:
                unemb.append(p)
            else:
                scalar.append(p)
        for params, lr, wd in ((emb, embedding_lr, weight_decay), (unemb, unembedding_lr, weight_decay),
                               (scalar, scalar_lr, 0.0)):
            for p in params:
                self.adamw.append({"p": p, "lr": lr, "wd": wd, "step": 0,
                                   "m": torch.zeros_like(p, dtype=torch.bfloat16),
                                   "v": torch.zeros_like(p, dtype=torch.bfloat16)})
        self.muon = []
        for (shape, split), params in sorted(muon.items(), key=lambda kv: str(kv[0])):
            rows, cols = shape
            parts = split or (rows,)
            self.muon.append({"params": params, "split": parts, "cols": cols, "lr": matrix_lr,
                              "wd": weight_decay, "momentum": 0.95,
                              "buf": torch.zeros(len(params), rows, cols, dtype=torch.bfloat16,
                                                 device=params[0].device)})
        self.lr_mult = 1.0

    def zero_grad(self) -> None:
        for g in self.adamw:
            g["p"].grad = None
        for g in self.muon:
            for p in g["params"]:
                p.grad = None

    @torch.no_grad()
    def step(self) -> None:
        for g in self.adamw:
            p = g["p"]
            if p.grad is None:
                continue
            g["step"] += 1
            lr = g["lr"] * self.lr_mult
            grad = p.grad.to(torch.bfloat16)
            p.mul_(1.0 - lr * g["wd"])
            g["m"].lerp_(grad, 0.1)
            g["v"].lerp_(grad.square(), 0.05)
            bc1 = 1.0 - 0.9 ** g["step"]
            bc2 = 1.0 - 0.95 ** g["step"]
            denom = (g["v"] / bc2).sqrt() + 1e-8
            p.add_((g["m"] / denom) * (lr / bc1), alpha=-1.0)
        for g in self.muon:
            params = [p for p in g["params"] if p.grad is not None]
            if len(params) != len(g["params"]):
                continue
            lr = g["lr"] * self.lr_mult
            mom = g["momentum"]
            grads = torch.stack([p.grad for p in params]).to(torch.bfloat16)
            buf = g["buf"]
            buf.lerp_(grads, 1.0 - mom)
            blend = grads.lerp(buf, mom)
            # split row blocks (q/k/v, gate/up) are orthogonalised separately
            pieces = torch.split(blend, list(g["split"]), dim=1)
            updates = []
            for piece in pieces:
                updates.append(newton_schulz5(piece))
            update = torch.cat(updates, dim=1)
            stacked = torch.stack(params)
            stacked.mul_(1.0 - lr * g["wd"])
            stacked.add_(update.to(stacked.dtype) * lr, alpha=-1.0)
            torch._foreach_copy_(params, list(stacked.unbind(0)))
