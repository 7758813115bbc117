"""The B200 operators under torch.compile: ``torch.library.opcheck`` on every custom
operator (schema, fake implementation against the real kernel, autograd
registration, AOT dispatch), and the model compiled the way the reference trains it
(kernels.py:126-137: ``fullgraph=True, dynamic=False``), forward and backward equal
to eager."""
from __future__ import annotations

import pytest
import torch

from parity import assert_bf16_close, assert_loss_close

pytestmark = pytest.mark.gpu


def _bf(g, *shape, std=1.0, grad=False, dev="cuda"):
    t = (torch.randn(*shape, generator=g) * std).to(torch.bfloat16).to(dev)
    return t.requires_grad_(grad)


def _op_cases(dev):
    from hackable_lm_b200 import ops

    g = torch.Generator().manual_seed(0)
    T, H, D, rd = 64, 2, 128, 32
    pos = torch.arange(T, dtype=torch.float32)
    inv = 1.0 / (10_000.0 ** (torch.arange(0, rd, 2, dtype=torch.float32) / rd))
    emb = torch.cat((torch.outer(pos, inv),) * 2, dim=-1)
    cos = emb.cos()[None, :, None, :].to(torch.bfloat16).to(dev)
    sin = emb.sin()[None, :, None, :].to(torch.bfloat16).to(dev)
    cos4, sin4 = cos.transpose(1, 2).contiguous(), sin.transpose(1, 2).contiguous()
    x = _bf(g, 2, T, 256, grad=True)
    w_qkv = _bf(g, 3 * H * D, 256, std=0.02, grad=True)
    q, k, v, rstd = ops.qkv_rope(x.detach(), w_qkv.detach(), cos4, sin4, H, H, 1e-6)
    gq, gk, gv = _bf(g, *q.shape), _bf(g, *k.shape), _bf(g, *v.shape)
    gate_up = _bf(g, 128, 512, grad=True)
    w_gu = _bf(g, 512, 256, std=0.02, grad=True)
    w_dn = _bf(g, 256, 256, std=0.02, grad=True)
    xm = _bf(g, 128, 256, grad=True)
    h, gu = ops.gate_up_swiglu(xm.detach(), w_gu.detach())
    hidden = _bf(g, 256, 128)
    w_head = _bf(g, 512, 128, std=0.02)
    targets = torch.randint(0, 512, (256,), generator=g).to(dev)
    targets[::17] = -1
    r, b = _bf(g, 4, 32, 384, grad=True), _bf(g, 4, 32, 384, grad=True)
    wn = (1 + 0.02 * torch.randn(384, generator=g)).to(dev).requires_grad_(True)
    return {
        "swiglu": (ops.swiglu, (gate_up,)),
        "swiglu_backward": (ops.swiglu_backward, (gate_up.detach(), _bf(g, 128, 256))),
        "gate_up_swiglu": (ops.gate_up_swiglu, (xm, w_gu)),
        "swiglu_down": (ops.swiglu_down, (h.detach().requires_grad_(True), gu.detach().requires_grad_(True), w_dn)),
        "swiglu_down_backward": (ops.swiglu_down_backward, (_bf(g, 128, 256), w_dn.detach(), gu.detach())),
        "rms_norm": (ops.rms_norm, (r, None, 1e-6)),
        "rms_norm_weighted": (ops.rms_norm, (r, wn, 1e-6)),
        "residual_rms_norm": (ops.residual_rms_norm, (r, b, None, 1e-6)),
        "rms_norm_backward": (ops.rms_norm_backward, (r.detach(), wn.detach(), b.detach(), r.detach(), 1e-6)),
        "qk_norm_rope": (ops.qk_norm_rope, (_bf(g, 2, T, H, D, grad=True), _bf(g, 2, T, H, D, grad=True),
                                            cos, sin, 1e-6)),
        "qk_norm_rope_backward": (ops.qk_norm_rope_backward, (q, k, gq, gk, cos, sin, 1e-6)),
        "qkv_rope": (ops.qkv_rope, (x, w_qkv, cos4, sin4, H, H, 1e-6)),
        "qkv_rope_backward": (ops.qkv_rope_backward, (x.detach(), w_qkv.detach(), q, k, rstd, cos4, sin4,
                                                      gq, gk, gv, H, H, 1e-6, True, True)),
        "lm_head_ce": (ops.lm_head_ce, (hidden, w_head, targets, -1, 0, True, True)),
        "scale_": (ops.scale_, (_bf(g, 1000), torch.tensor(0.25, device=dev))),
        "proj_residual_norm": (ops.proj_residual_norm, (_bf(g, 256, 256, grad=True), _bf(g, 768, 256, std=0.02, grad=True),
                                                        _bf(g, 256, 768, grad=True), 1e-6)),
        "swiglu_down_residual_norm": (ops.swiglu_down_residual_norm,
                                      (h.detach().requires_grad_(True), gu.detach().requires_grad_(True),
                                       _bf(g, 256, 256, std=0.02, grad=True), _bf(g, 128, 256, grad=True), 1e-6)),
    }


OP_NAMES = ["swiglu", "swiglu_backward", "gate_up_swiglu", "swiglu_down", "swiglu_down_backward", "rms_norm", "rms_norm_weighted",
            "residual_rms_norm", "rms_norm_backward", "qk_norm_rope", "qk_norm_rope_backward", "qkv_rope",
            "qkv_rope_backward", "lm_head_ce", "scale_", "proj_residual_norm", "swiglu_down_residual_norm"]


@pytest.mark.parametrize("name", OP_NAMES)
def test_opcheck(name, cuda_device):
    op, args = _op_cases(cuda_device)[name]
    torch.library.opcheck(op, args)


def test_compiled_model_matches_eager(cuda_device):
    """Depth-2 B200 model: torch.compile(fullgraph=True, dynamic=False) forward and
    backward against the same model run eagerly (same weights, same batch)."""
    from hackable_lm_b200 import config as hcfg
    from hackable_lm_b200 import kernels
    from hackable_lm_b200.model import LanguageModel

    torch.manual_seed(0)
    cfg = hcfg.model_config_for_depth(2, vocab_size=4096, sequence_len=256, attention_window=64, backend="b200")
    eager = LanguageModel(cfg).to(cuda_device)
    kernels.apply_precision_policy(eager, "bf16")
    twin = LanguageModel(cfg).to(cuda_device)
    kernels.apply_precision_policy(twin, "bf16")
    twin.load_state_dict(eager.state_dict())
    compiled = kernels.compile_training_model(twin, True)
    g = torch.Generator().manual_seed(2)
    ids = torch.randint(0, 4096, (2, 257), generator=g).to(cuda_device)
    x, y = ids[:, :-1], ids[:, 1:]
    _, le = eager(x, y)
    (le / 4).backward()
    for _ in range(2):  # second call runs the cached graph
        twin.zero_grad(set_to_none=True)
        _, lc = compiled(x, y)
        (lc / 4).backward()
    torch.cuda.synchronize()
    assert_loss_close(lc.detach(), le.detach(), tol=1e-4, what="compiled loss")
    pe = dict(eager.named_parameters())
    for n, p in twin.named_parameters():
        assert_bf16_close(p.grad, pe[n].grad, what=f"compiled grad {n}")
