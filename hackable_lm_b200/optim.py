"""Muon + AdamW optimizer step for the data-parallel training step, with the Muon
work sharded across data-parallel ranks.

The update rule restates the reference's MuonAdamW (optim.py:20-75, 170-262,
313-329, 403-452):

* AdamW (betas 0.9/0.95, eps 1e-8, bf16 moments) for the token embedding and the
  LM head (optim.py:20-43, 102-139);
* Muon for the 2-D block matrices, grouped by shape, with qkv_proj split into its
  q/k/v row blocks and gate_up_proj into gate/up halves (optim.py:387-399,
  434-452): bf16 momentum lerp, Nesterov-style blend, Frobenius normalisation,
  five quintic Newton-Schulz iterations with coefficients (3.4445, -4.7750,
  2.0315), decoupled weight decay and the update (optim.py:46-75).  The
  reference casts momentum to the bf16 state dtype and lr / weight decay to the
  parameter dtype before using them (optim.py:53, 72-74); so does this step.

Sharding (the part that differs from the reference, which runs the whole step on
every rank): a Muon group of n matrices is cut into contiguous per-rank slices
of ceil(n / world) matrices.  Each rank keeps the momentum of its own slice only,
runs the Newton-Schulz iterations on it (one batched call per group: the equal
q/k/v or gate/up row blocks are viewed as a batch of square-ish blocks), applies
weight decay and the update to its slice, and one all-gather of all groups'
updated bf16 matrices (a single flat buffer) gives every rank the full,
identical parameters.  The Newton-Schulz cost per rank falls as 1/world; the
all-gather moves the Muon parameters once (226 MB of bf16 at depth 12).  With
one rank (or no process group) nothing is gathered and the step equals the
replicated reference step.
"""
from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist

MUON_NAME_MARKERS = ("qkv_proj.weight", "o_proj.weight", "gate_up_proj.weight", "down_proj.weight")
NS_COEFFS = (3.4445, -4.7750, 2.0315)


def _bf16(x: float) -> float:
    """x rounded to bf16 (the reference's scalar casts, optim.py:53, 72-73)."""
    return float(torch.tensor(x, dtype=torch.float32).to(torch.bfloat16))


def _f32(x: float) -> float:
    """x rounded to fp32 (the reference keeps optimizer scalars in fp32 tensors, optim.py:17)."""
    return float(torch.tensor(x, dtype=torch.float32))


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


def _orthogonalise(blend: torch.Tensor, split: tuple[int, ...]) -> torch.Tensor:
    """Newton-Schulz on each row block of every stacked matrix: [n, rows, cols] with
    rows cut into ``split``.  Equal blocks run as one batch of n * len(split)."""
    n, rows, cols = blend.shape
    if len(set(split)) == 1:
        return newton_schulz5(blend.reshape(n * len(split), split[0], cols)).reshape(n, rows, cols)
    return torch.cat([newton_schulz5(piece) for piece in torch.split(blend, list(split), dim=1)], dim=1)


class MuonAdamW:
    def __init__(self, model: torch.nn.Module, *, embedding_lr: float, unembedding_lr: float,
                 matrix_lr: float, scalar_lr: float, weight_decay: float, n_head: int, n_kv_head: int,
                 head_dim: int, process_group: Any = None, shard: bool = True) -> None:
        distributed = dist.is_available() and dist.is_initialized()
        self.group = process_group
        self.world = dist.get_world_size(process_group) if (distributed and shard) else 1
        self.rank = dist.get_rank(process_group) if (distributed and shard) else 0
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
        gather_elems = 0
        for (shape, split), params in sorted(muon.items(), key=lambda kv: str(kv[0])):
            rows, cols = shape
            n = len(params)
            chunk = -(-n // self.world)
            own = list(range(min(n, self.rank * chunk), min(n, (self.rank + 1) * chunk)))
            self.muon.append({"params": params, "split": split or (rows,), "rows": rows, "cols": cols,
                              "lr": matrix_lr, "wd": weight_decay, "momentum": 0.95, "own": own,
                              "chunk": chunk, "offset": gather_elems,
                              "buf": torch.zeros(len(own), rows, cols, dtype=torch.bfloat16,
                                                 device=params[0].device)})
            gather_elems += chunk * rows * cols
        self.gather_elems = gather_elems  # per rank
        self._send: torch.Tensor | None = None
        self._recv: torch.Tensor | None = None
        self.lr_mult = 1.0

    def zero_grad(self) -> None:
        for g in self.adamw:
            g["p"].grad = None
        for g in self.muon:
            for p in g["params"]:
                p.grad = None

    def parameters(self) -> list[torch.nn.Parameter]:
        return [g["p"] for g in self.adamw] + [p for g in self.muon for p in g["params"]]

    @torch.no_grad()
    def _step_adamw(self) -> None:
        for g in self.adamw:
            p = g["p"]
            if p.grad is None:
                continue
            g["step"] += 1
            # fp32 scalars as the reference's 0-d fp32 tensors give them (optim.py:120-139)
            lr, wd = _f32(g["lr"] * self.lr_mult), _f32(g["wd"])
            b1, b2 = _f32(0.9), _f32(0.95)
            grad = p.grad.to(torch.bfloat16)
            p.mul_(_f32(1.0 - _f32(lr * wd)))
            g["m"].lerp_(grad, _f32(1.0 - b1))
            g["v"].lerp_(grad.square(), _f32(1.0 - b2))
            bc1 = _f32(1.0 - _f32(b1 ** g["step"]))
            bc2 = _f32(1.0 - _f32(b2 ** g["step"]))
            denom = (g["v"] / bc2).sqrt() + _f32(1e-8)
            p.add_((g["m"] / denom) * _bf16(_f32(lr / bc1)), alpha=-1.0)

    @torch.no_grad()
    def _muon_update(self, g: dict[str, Any]) -> torch.Tensor | None:
        """Momentum, Newton-Schulz, weight decay and update of this rank's slice of a
        group; returns the updated slice [len(own), rows, cols] (bf16)."""
        params, own = g["params"], g["own"]
        if not own:
            return None
        mom = _bf16(g["momentum"])
        lr = _bf16(g["lr"] * self.lr_mult)
        decay = _bf16(1.0 - _bf16(lr * _bf16(g["wd"])))
        grads = torch.stack([params[i].grad for i in own]).to(torch.bfloat16)
        buf = g["buf"]
        buf.lerp_(grads, 1.0 - mom)
        blend = grads.lerp(buf, mom)
        update = _orthogonalise(blend, tuple(g["split"]))
        stacked = torch.stack([params[i] for i in own])
        stacked.mul_(decay)
        stacked.add_(update.to(stacked.dtype) * lr, alpha=-1.0)
        return stacked

    @torch.no_grad()
    def step(self) -> None:
        self._step_adamw()
        groups = [g for g in self.muon if all(p.grad is not None for p in g["params"])]
        if self.world == 1:
            for g in groups:
                stacked = self._muon_update(g)
                torch._foreach_copy_(g["params"], list(stacked.unbind(0)))
            return
        if len(groups) != len(self.muon):
            raise RuntimeError("sharded Muon step: every Muon parameter needs a gradient on every rank")
        if self._send is None:
            dev, dt = self.muon[0]["params"][0].device, self.muon[0]["params"][0].dtype
            self._send = torch.zeros(self.gather_elems, dtype=dt, device=dev)
            self._recv = torch.empty(self.world * self.gather_elems, dtype=dt, device=dev)
        for g in self.muon:
            stacked = self._muon_update(g)
            if stacked is not None:
                n_own = len(g["own"]) * g["rows"] * g["cols"]
                self._send[g["offset"]:g["offset"] + n_own].copy_(stacked.reshape(-1))
        dist.all_gather_into_tensor(self._recv, self._send, group=self.group)
        recv = self._recv.view(self.world, self.gather_elems)
        dst, src = [], []
        for g in self.muon:
            rows, cols, chunk = g["rows"], g["cols"], g["chunk"]
            per_rank = recv[:, g["offset"]:g["offset"] + chunk * rows * cols].reshape(self.world * chunk, rows, cols)
            dst.extend(g["params"])
            src.extend(per_rank[:len(g["params"])].unbind(0))
        torch._foreach_copy_(dst, src)
