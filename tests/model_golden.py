"""Helpers for the whole-model golden fixtures (``tests/golden/model_*.pt``), which
``tests/golden/make_golden.py`` made by running the reference's own LanguageModel:
re-create the same weights from the fixture's seed with this package's model and
compare a forward + backward with the stored loss and gradients."""
from __future__ import annotations

import torch

from hackable_lm_b200 import config as hcfg
from hackable_lm_b200.model import LanguageModel


def fingerprint(t: torch.Tensor) -> torch.Tensor:
    """Same summary as make_golden.py's: sum, abs-sum, first and last 8 elements."""
    flat = t.detach().reshape(-1).double()
    return torch.stack([flat.sum(), flat.abs().sum(), flat[:8].sum(), flat[-8:].sum()])


def build(gd: dict, backend: str, attention_backend: str | None = None) -> LanguageModel:
    """This package's LanguageModel with the fixture's dimensions, initialised from the
    fixture's seed on the CPU in fp32 (the reference's init order, model.py:370-380),
    checked against the stored init fingerprints, then rounded to bf16 values.  The
    attention core defaults to SDPA with the b200 operators and to the explicit
    softmax with the torch ones."""
    c = gd["config"]
    if attention_backend is None:
        attention_backend = "sdpa" if backend == "b200" else "torch"
    cfg = hcfg.model_config_for_depth(c["depth"], vocab_size=c["vocab"], sequence_len=c["seq"],
                                      attention_window=c["window"], backend=backend,
                                      attention_backend=attention_backend)
    assert (cfg.n_embd, cfg.n_head, cfg.mlp_hidden, cfg.attention_full_every, cfg.loss_chunk_size) == (
        c["n_embd"], c["n_head"], c["mlp_hidden"], c["attention_full_every"], c["loss_chunk_size"])
    assert (cfg.rope_theta, cfg.rope_fraction) == (c["rope_theta"], c["rope_fraction"])
    torch.manual_seed(gd["seed"])
    model = LanguageModel(cfg)
    fps = gd["init_fingerprint"]
    assert set(fps) == {n for n, _ in model.named_parameters()}
    for n, p in model.named_parameters():
        # the fp64 sums depend on the reduction order (thread count) in the last bits only;
        # a different init would differ in every digit
        got, ref = fingerprint(p), fps[n]
        assert ((got - ref).abs() <= 1e-9 * (ref[1].abs() + 1.0)).all(), f"init of {n} differs from the reference's"
    with torch.no_grad():
        for p in model.parameters():
            p.copy_(p.to(torch.bfloat16).float())
    return model


def batch(gd: dict, device) -> tuple[torch.Tensor, torch.Tensor]:
    ids = gd["ids"].to(device)
    return ids[:, :-1], ids[:, 1:]


def grad_errors(model: torch.nn.Module, gd: dict) -> dict[str, tuple[float, float]]:
    """Per parameter: (relative error of the gradient norm, max |err| / rms over the
    stored gradient rows)."""
    out = {}
    for n, p in model.named_parameters():
        g = p.grad.detach().double().cpu()
        ref_norm = gd["grad_norm"][n].item()
        rows, ref_rows = gd["grad_rows"][n]
        got = g[rows]
        ref = ref_rows.double()
        rms = ref.pow(2).mean().sqrt().item()
        out[n] = (abs(g.norm().item() - ref_norm) / ref_norm, (got - ref).abs().max().item() / rms)
    return out
