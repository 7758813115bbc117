"""Generate the golden fixtures in this directory by running the REFERENCE's own
CPU implementation of every hot-path operator (hackable-lm's kernels.py /
model.py imported from a checkout of the reference repository).

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --reference /path/to/hackable-lm

The fixtures pin the CPU oracle (oracle/hotpath.py); the GPU parity tests
then compare the CUDA kernels against the pinned oracle.  Inputs are seeded
(torch.Generator().manual_seed(0)) and generated on the CPU in fp32; the
fixtures whose GPU tests feed bf16 inputs (qkv, lm_head, the model cases) hold
bf16-representable values.  The model cases (model_d4_window, model_d12) run
the reference's whole LanguageModel.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent


def gen(seed: int = 0) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def randn(g, *shape, std=1.0, mean=0.0):
    return torch.randn(*shape, generator=g) * std + mean


def bf16_values(t: torch.Tensor) -> torch.Tensor:
    """fp32 tensor holding bf16-representable values: the fixtures whose GPU tests feed
    bf16 inputs use them, so both sides start from identical numbers."""
    return t.to(torch.bfloat16).to(torch.float32)


def fingerprint(t: torch.Tensor) -> torch.Tensor:
    flat = t.detach().reshape(-1).double()
    return torch.stack([flat.sum(), flat.abs().sum(), flat[:8].sum(), flat[-8:].sum()])


def make_rmsnorm_c1(model):
    # x, residual [4,256,384] ~ N(0,1); weight = 1 + N(0, 0.02);
    # eps 1e-6; upstream grad ~ N(0,1); seed 0; fp32 on CPU.
    g = gen(0)
    x = randn(g, 4, 256, 384)
    residual = randn(g, 4, 256, 384)
    weight = 1.0 + randn(g, 384, std=0.02)
    grad = randn(g, 4, 256, 384)
    xr = x.clone().requires_grad_(True)
    rr = residual.clone().requires_grad_(True)
    wr = weight.clone().requires_grad_(True)
    out = rr + xr  # model.residual_rms_norm's add (model.py:74)
    norm = model.rms_norm_torch(out, wr, 1e-6)
    norm.backward(grad)
    rows = torch.randperm(1024, generator=gen(1))[:64]
    flat = lambda t: t.detach().reshape(1024, 384)[rows].clone()  # noqa: E731
    return {
        "fingerprint": {"x": fingerprint(x), "residual": fingerprint(residual),
                        "weight": fingerprint(weight), "grad": fingerprint(grad)},
        "rows": rows,
        "out": flat(out), "norm": flat(norm), "grad_x": flat(xr.grad),
        "grad_residual": flat(rr.grad), "grad_weight": wr.grad.detach().clone(), "eps": 1e-6,
    }


def make_residual_rms_norm(model):
    g = gen(0)
    residual = randn(g, 2, 8, 64)
    branch = randn(g, 2, 8, 64)
    g_out = randn(g, 2, 8, 64)
    g_norm = randn(g, 2, 8, 64)
    rr = residual.clone().requires_grad_(True)
    br = branch.clone().requires_grad_(True)
    out, norm = model.residual_rms_norm(rr, br, 1e-6)
    ((out * g_out).sum() + (norm * g_norm).sum()).backward()
    return {"residual": residual, "branch": branch, "grad_out": g_out, "grad_norm": g_norm,
            "out": out.detach(), "norm": norm.detach(), "grad_residual": rr.grad, "grad_branch": br.grad,
            "eps": 1e-6}


def make_swiglu(kernels):
    cases = []
    for shape in ((2, 5, 64), (17, 130), (4, 512)):
        g = gen(0)
        gate_up = randn(g, *shape)
        grad = randn(g, *shape[:-1], shape[-1] // 2)
        x = gate_up.clone().requires_grad_(True)
        out = kernels.swiglu_triton(x)  # CPU branch (kernels.py:752-753)
        out.backward(grad)
        cases.append({"gate_up": gate_up, "grad_out": grad, "out": out.detach(), "grad_gate_up": x.grad})
    return {"cases": cases}


def make_rope_tables(model):
    out = []
    for theta, fraction, T in ((1_000_000.0, 0.25, 64), (10_000.0, 0.25, 64), (10_000.0, 1.0, 64)):
        rope = model.RotaryEmbedding(128, theta, fraction)
        cos, sin = rope(T, torch.device("cpu"), torch.float32)
        out.append({"theta": theta, "fraction": fraction, "T": T, "cos": cos.clone(), "sin": sin.clone()})
    return {"cases": out}


def make_qk_norm_rope(kernels, model):
    cases = []
    # the reference's own unit-test shape (GQA, rotary_dim 4 from random freqs)
    g = gen(0)
    q = randn(g, 2, 5, 3, 8)
    k = randn(g, 2, 5, 2, 8)
    freqs = randn(g, 5, 2)
    cos = torch.cat((freqs.cos(), freqs.cos()), dim=-1)[None, :, None, :]
    sin = torch.cat((freqs.sin(), freqs.sin()), dim=-1)[None, :, None, :]
    cases.append((q, k, cos, sin))
    # model-shaped: head_dim 128 with the model's tables (fraction 0.25 and 1.0)
    for fraction in (0.25, 1.0):
        g = gen(0)
        q = randn(g, 2, 16, 2, 128)
        k = randn(g, 2, 16, 2, 128)
        c, s = model.RotaryEmbedding(128, 10_000.0, fraction)(16, torch.device("cpu"), torch.float32)
        cases.append((q, k, c.transpose(1, 2), s.transpose(1, 2)))
    out = []
    for q, k, cos, sin in cases:
        g = gen(2)
        dq = randn(g, *q.shape)
        dk = randn(g, *k.shape)
        qr = q.clone().requires_grad_(True)
        kr = k.clone().requires_grad_(True)
        qo, ko = kernels.qk_norm_rope_triton(qr, kr, cos, sin, 1e-6)  # CPU branch (kernels.py:766-771)
        ((qo * dq).sum() + (ko * dk).sum()).backward()
        out.append({"q": q, "k": k, "cos": cos, "sin": sin, "grad_q_out": dq, "grad_k_out": dk,
                    "q_out": qo.detach(), "k_out": ko.detach(), "grad_q": qr.grad, "grad_k": kr.grad,
                    "eps": 1e-6})
    return {"cases": out}


def make_qkv(model, config):
    cfg = config.ModelConfig(vocab_size=64, block_size=16, n_layer=1, n_embd=256, n_head=2, n_kv_head=2,
                             rope_theta=10_000.0, rope_fraction=0.25, qkv_backend="torch")
    mod = model.QKVProjection(cfg, 0)
    g = gen(0)
    with torch.no_grad():
        mod.qkv_proj.weight.copy_(bf16_values(randn(g, *mod.qkv_proj.weight.shape, std=0.02)))
    x = bf16_values(randn(g, 2, 16, 256))
    xr = x.clone().requires_grad_(True)
    q, k, v = mod.fwd_torch(xr)  # model.py:101-115
    g2 = gen(3)
    dq, dk, dv = (bf16_values(randn(g2, *t.shape)) for t in (q, k, v))
    ((q * dq).sum() + (k * dk).sum() + (v * dv).sum()).backward()
    cos, sin = mod.rope(16, torch.device("cpu"), torch.float32)
    return {"x": x, "w_qkv": mod.qkv_proj.weight.detach().clone(), "cos": cos.clone(), "sin": sin.clone(),
            "n_head": 2, "n_kv_head": 2, "eps": cfg.norm_eps, "q": q.detach(), "k": k.detach(),
            "v": v.detach(), "grad_q_out": dq, "grad_k_out": dk, "grad_v_out": dv, "grad_x": xr.grad,
            "grad_w": mod.qkv_proj.weight.grad.detach().clone()}


def make_lm_head(kernels, model, config):
    out = {}
    # chunked module path (model.py:325-339), no ignored targets
    cfg = config.ModelConfig(vocab_size=96, block_size=7, n_layer=1, n_embd=64, n_head=1, n_kv_head=1,
                             loss_chunk_size=8, lm_head_backend="torch")
    head = model.LMHeadProjection(cfg)
    g = gen(0)
    with torch.no_grad():
        head.lm_head.weight.copy_(randn(g, 96, 64, std=0.02))
    hidden = randn(g, 3, 7, 64)
    targets = torch.randint(0, 96, (3, 7), generator=g)
    hr = hidden.clone().requires_grad_(True)
    _, loss = head(hr, targets)
    loss.backward()
    out["chunked"] = {"hidden": hidden, "weight": head.lm_head.weight.detach().clone(), "targets": targets,
                      "chunk": 8, "loss": loss.detach(), "grad_hidden": hr.grad,
                      "grad_weight": head.lm_head.weight.grad.detach().clone(), "ignore_index": -100}
    # dense CPU branch of fused_linear_cross_entropy_with_weight (kernels.py:955-957) with some
    # targets set to F.cross_entropy's ignore_index: mean over the non-ignored rows.
    g = gen(1)
    w = bf16_values(randn(g, 96, 64, std=0.02))
    hidden = bf16_values(randn(g, 40, 64))
    targets = torch.randint(0, 96, (40,), generator=g)
    targets[torch.randperm(40, generator=g)[:5]] = -100
    hr = hidden.clone().requires_grad_(True)
    wr = w.clone().requires_grad_(True)
    loss = kernels.fused_linear_cross_entropy_with_weight(hr, wr, None, targets, "triton")
    loss.backward()
    out["dense_ignore"] = {"hidden": hidden, "weight": w, "targets": targets, "loss": loss.detach(),
                           "grad_hidden": hr.grad, "grad_weight": wr.grad, "ignore_index": -100}
    return out


MODEL_CASES = {
    # depth 4 with sliding windows (layers 0-2 windowed, layer 3 full: every fourth
    # and the last layer attend to the whole sequence, config.py:184-191)
    "model_d4_window": dict(depth=4, vocab=4096, seq=256, batch=2, window=64, seed=0, rows=16),
    # BASELINE config 5's model: depth 12, vocab 32768, seq 2048, full causal
    "model_d12": dict(depth=12, vocab=32768, seq=2048, batch=1, window=None, seed=0, rows=6),
}


def make_model(model, config, *, depth, vocab, seq, batch, window, seed, rows):
    """The reference LanguageModel (model.py:355-391) built by the reference's own
    resolve_config (config.py:289-488), seeded GPT-style init, then every weight
    rounded to bf16 (the B200 model trains in bf16, kernels.py:962-972) and one
    forward + backward on the CPU in fp32 with the torch backends.

    Stored: the init fingerprints (before rounding; a test re-creating the weights
    from the same seed checks them), the token ids, the loss, every parameter's
    gradient norm and a seeded subset of gradient rows per parameter (for the token
    embedding, rows of ids present in the batch)."""
    resolved = config.resolve_config(depth=depth, vocab_size=vocab, sequence_len=seq, device_batch_size=batch,
                                     attention_window=window, attention_backend="torch", qkv_backend="torch",
                                     gate_up_backend="torch", lm_head_backend="torch")
    cfg = resolved.model
    torch.manual_seed(seed)
    m = model.LanguageModel(cfg)
    fps = {n: fingerprint(p) for n, p in m.named_parameters()}
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(bf16_values(p))
    ids = torch.randint(0, vocab, (batch, seq + 1), generator=gen(seed + 1))
    x, y = ids[:, :-1], ids[:, 1:]
    _, loss = m(x, y)
    loss.backward()
    used = torch.unique(x)
    grad_norms, grad_rows = {}, {}
    for i, (n, p) in enumerate(m.named_parameters()):
        grad = p.grad.detach()
        grad_norms[n] = grad.double().norm()
        pool = used if n == "tok_emb.weight" else torch.arange(p.shape[0])
        pick = pool[torch.randperm(pool.numel(), generator=gen(100 + i))[:rows]]
        grad_rows[n] = (pick.clone(), grad[pick].clone())
    return {"config": dict(depth=depth, vocab=vocab, seq=seq, batch=batch, window=window,
                           attention_full_every=cfg.attention_full_every, n_embd=cfg.n_embd,
                           n_head=cfg.n_head, mlp_hidden=cfg.mlp_hidden, rope_theta=cfg.rope_theta,
                           rope_fraction=cfg.rope_fraction, loss_chunk_size=cfg.loss_chunk_size),
            "seed": seed, "init_fingerprint": fps, "ids": ids, "loss": loss.detach().double(),
            "grad_norm": grad_norms, "grad_rows": grad_rows}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("HACKABLE_LM_REFERENCE"),
                    required="HACKABLE_LM_REFERENCE" not in os.environ,
                    help="path of the hackable-lm checkout (default: $HACKABLE_LM_REFERENCE)")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--only", nargs="*", help="fixture names to write (default: all)")
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference)
    import config  # noqa: E402  (the reference's modules)
    import kernels  # noqa: E402
    import model  # noqa: E402

    torch.set_num_threads(max(1, torch.get_num_threads()))
    makers = {
        "rmsnorm_c1": lambda: make_rmsnorm_c1(model),
        "residual_rms_norm": lambda: make_residual_rms_norm(model),
        "swiglu": lambda: make_swiglu(kernels),
        "rope_tables": lambda: make_rope_tables(model),
        "qk_norm_rope": lambda: make_qk_norm_rope(kernels, model),
        "qkv": lambda: make_qkv(model, config),
        "lm_head": lambda: make_lm_head(kernels, model, config),
    }
    for name, case in MODEL_CASES.items():
        makers[name] = lambda case=case: make_model(model, config, **case)
    outdir = Path(args.out)
    for name, make in makers.items():
        if args.only and name not in args.only:
            continue
        path = outdir / f"{name}.pt"
        torch.save(make(), path)
        print(f"wrote {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
