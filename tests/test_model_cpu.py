"""The model's reference ("torch") backend against the oracle restatement of the
reference decoder, and the optimizer's Newton-Schulz step, on the CPU."""
from __future__ import annotations

import torch

from hackable_lm_b200 import config as hcfg
from hackable_lm_b200.model import LanguageModel
from hackable_lm_b200.optim import MuonAdamW, newton_schulz5


def tiny_config(**kw):
    base = dict(vocab_size=64, sequence_len=16, backend="torch", attention_backend="torch")
    base.update(kw)
    return hcfg.model_config_for_depth(2, **base)


def test_parameter_names_match_reference_layout():
    model = LanguageModel(tiny_config())
    names = {n for n, _ in model.named_parameters()}
    for want in ("tok_emb.weight", "blocks.0.attn.qkv.qkv_proj.weight", "blocks.0.attn.out.o_proj.weight",
                 "blocks.1.mlp.gate_up.gate_up_proj.weight", "blocks.1.mlp.down.down_proj.weight",
                 "lm_head.lm_head.weight"):
        assert want in names
    d12 = hcfg.model_config_for_depth(12)
    assert LanguageModel(d12).parameter_count() == 135_266_304


def test_torch_backend_matches_oracle_model():
    from oracle import model as om

    cfg = tiny_config()
    torch.manual_seed(0)
    model = LanguageModel(cfg)
    p = {"tok_emb": model.tok_emb.weight.detach().clone(), "lm_head": model.lm_head.lm_head.weight.detach().clone()}
    for i, blk in enumerate(model.blocks):
        p[f"{i}.qkv"] = blk.attn.qkv.qkv_proj.weight.detach().clone()
        p[f"{i}.o"] = blk.attn.out.o_proj.weight.detach().clone()
        p[f"{i}.gate_up"] = blk.mlp.gate_up.gate_up_proj.weight.detach().clone()
        p[f"{i}.down"] = blk.mlp.down.down_proj.weight.detach().clone()
    g = torch.Generator().manual_seed(1)
    ids = torch.randint(0, 64, (2, 17), generator=g)
    x, y = ids[:, :-1], ids[:, 1:]
    _, loss = model(x, y)
    ref = om.forward_loss(p, x, y, n_layer=2, n_head=cfg.n_head, head_dim=cfg.head_dim,
                          rope_theta=cfg.rope_theta, rope_fraction=cfg.rope_fraction, loss_chunk=cfg.loss_chunk_size)
    torch.testing.assert_close(loss, ref, atol=1e-5, rtol=1e-5)


def test_newton_schulz_orthogonalises():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(3, 48, 32, generator=g)
    y = newton_schulz5(x).float()
    # singular values are pushed towards ~1 (the quintic's fixed band is roughly [0.7, 1.2])
    s = torch.linalg.svdvals(y)
    assert s.min() > 0.5 and s.max() < 1.3


def test_optimizer_updates_every_parameter():
    cfg = tiny_config()
    torch.manual_seed(0)
    model = LanguageModel(cfg)
    opt = MuonAdamW(model, embedding_lr=0.1, unembedding_lr=0.01, matrix_lr=0.02, scalar_lr=0.1,
                    weight_decay=0.1, n_head=cfg.n_head, n_kv_head=cfg.n_kv_head, head_dim=cfg.head_dim)
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    ids = torch.randint(0, 64, (2, 17))
    _, loss = model(ids[:, :-1], ids[:, 1:])
    loss.backward()
    opt.step()
    for n, p in model.named_parameters():
        assert not torch.equal(before[n], p.detach()), n


def test_torch_backend_matches_reference_model_fixture(golden):
    """This package's model (reference formulation, fp32, CPU) against the reference's
    own LanguageModel on the same seeded weights and batch (depth 4, windowed
    attention): init fingerprints, loss and gradients agree to fp32 rounding."""
    import model_golden as mg

    gd = golden("model_d4_window")
    model = mg.build(gd, "torch")
    x, y = mg.batch(gd, "cpu")
    _, loss = model(x, y)
    loss.backward()
    assert abs(loss.item() - gd["loss"].item()) <= 1e-5 * gd["loss"].item()
    for n, (norm_err, row_err) in mg.grad_errors(model, gd).items():
        assert norm_err <= 1e-4 and row_err <= 1e-4, (n, norm_err, row_err)


def test_b200_model_traces_fullgraph_on_meta():
    """The B200 model compiles the way the reference trains (torch.compile with
    fullgraph=True, dynamic=False, kernels.py:126-137) with no graph break, forward and
    backward: traced on meta tensors (the operators' fake implementations) with the
    aot_eager backend, every B200 operator of the step appears in the graph.  The GPU
    test runs the compiled model against eager."""
    from torch.utils._python_dispatch import TorchDispatchMode

    from hackable_lm_b200 import kernels

    class Rec(TorchDispatchMode):
        def __init__(self):
            super().__init__()
            self.ops = set()

        def __torch_dispatch__(self, func, types, args=(), kwargs=None):
            self.ops.add(str(func.overloadpacket))
            return func(*args, **(kwargs or {}))

    cfg = hcfg.model_config_for_depth(2, vocab_size=4096, sequence_len=256, attention_window=64, backend="b200")
    with torch.device("meta"):
        m = LanguageModel(cfg)
    kernels.apply_precision_policy(m, "bf16")
    compiled = torch.compile(m, backend="aot_eager", fullgraph=True, dynamic=False)
    ids = torch.randint(0, 4096, (2, 256), device="meta")
    rec = Rec()
    with rec:
        _, loss = compiled(ids, ids)
        loss.backward()
    want = {f"hackable_lm_b200.{n}" for n in (
        "qkv_rope", "qkv_rope_backward", "gate_up_swiglu", "swiglu_down_residual_norm", "swiglu_down_backward",
        "proj_residual_norm", "rms_norm", "rms_norm_backward", "lm_head_ce", "scale_")}
    assert not want - rec.ops, sorted(want - rec.ops)
    for n, p in m.named_parameters():
        assert p.grad is not None and p.grad.shape == p.shape, n
