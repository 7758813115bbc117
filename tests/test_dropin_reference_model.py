"""The reference's own model.py, unmodified, running on this package's kernels module.

The reference ``LanguageModel`` imports a module named ``kernels`` and calls its
entry points: ``qk_norm_rope_triton``, ``swiglu_triton``,
``fused_linear_cross_entropy_with_weight``, ``scaled_dot_product_attention`` and
``flex_attention_block_mask`` (model.py:117-126, 160-251, 291-292, 341-352).  Here
``hackable_lm_b200.kernels`` is installed under that name, the reference model is
built from the reference's own ``config.resolve_config`` with its default backends
(triton modules, flash_attn_2 attention, 512-token windows every layer but every
fourth and the last) on the meta device, and run forward and backward.  A dispatch
mode records every operator that runs: the B200 custom operators must be among
them (on meta tensors they run their fake implementations, which carry the shapes;
the CUDA kernels behind them are covered by the GPU tests).  The numerical side of
the same swap is pinned by the GPU test against the golden fixtures that
``tests/golden/make_golden.py`` made from this reference model.

Needs a reference checkout (``HACKABLE_LM_REFERENCE`` or a ``reference`` /
``hackable-lm`` directory beside the repository); skipped without one.
"""
from __future__ import annotations

import sys

import pytest
import torch
from torch.utils._python_dispatch import TorchDispatchMode

from conftest import reference_checkout

REF = reference_checkout()
pytestmark = pytest.mark.skipif(REF is None, reason="no hackable-lm reference checkout")


class _Recorder(TorchDispatchMode):
    def __init__(self):
        super().__init__()
        self.ops: set[str] = set()

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        self.ops.add(str(func.overloadpacket))
        return func(*args, **(kwargs or {}))


@pytest.fixture()
def reference_modules():
    """The reference's config and model modules, importing hackable_lm_b200.kernels as
    ``kernels``; sys.modules and sys.path are restored afterwards."""
    import hackable_lm_b200.kernels as b200_kernels

    names = ("config", "model", "kernels")
    saved = {n: sys.modules.pop(n) for n in names if n in sys.modules}
    saved_path = list(sys.path)
    dont_write = sys.dont_write_bytecode
    sys.dont_write_bytecode = True
    sys.modules["kernels"] = b200_kernels
    sys.path.insert(0, str(REF))
    try:
        import config as ref_config
        import model as ref_model

        assert ref_model.kernels is b200_kernels
        yield ref_config, ref_model
    finally:
        for n in names:
            sys.modules.pop(n, None)
        sys.modules.update(saved)
        sys.path[:] = saved_path
        sys.dont_write_bytecode = dont_write


B200_OPS = {"hackable_lm_b200.qk_norm_rope", "hackable_lm_b200.swiglu", "hackable_lm_b200.lm_head_ce",
            "hackable_lm_b200.qk_norm_rope_backward", "hackable_lm_b200.swiglu_backward",
            "hackable_lm_b200.scale_"}


@pytest.mark.parametrize("attention_backend", ["flash_attn_2", "flex_attention"])
def test_reference_model_runs_on_b200_kernels(reference_modules, attention_backend):
    ref_config, ref_model = reference_modules
    from hackable_lm_b200 import kernels

    resolved = ref_config.resolve_config(depth=4, vocab_size=1024, sequence_len=256, device_batch_size=2,
                                         attention_window=64, attention_backend=attention_backend)
    cfg = resolved.model
    assert (cfg.qkv_backend, cfg.gate_up_backend, cfg.lm_head_backend) == ("triton",) * 3
    with torch.device("meta"):
        m = ref_model.LanguageModel(cfg)
    kernels.apply_precision_policy(m, "bf16")
    # the reference's AttentionCore picks "torch" only for CPU tensors (model.py:169)
    idx = torch.randint(0, 1024, (2, 256), device="meta")
    tgt = torch.randint(0, 1024, (2, 256), device="meta")
    rec = _Recorder()
    with rec:
        _, loss = m(idx, tgt)
        loss.backward()
    assert loss.shape == () and loss.dtype == torch.float32
    missing = B200_OPS - rec.ops
    assert not missing, f"reference model did not reach {sorted(missing)}; ran {sorted(rec.ops)}"
    for n, p in m.named_parameters():
        assert p.grad is not None and p.grad.shape == p.shape and p.grad.dtype == torch.bfloat16, n


def test_reference_attention_calls_accepted(reference_modules):
    """The reference's attention call forms (model.py:176-251) on this module: the
    FlashAttention names take [B, T, H, D], flex_attention a block mask from
    flex_attention_block_mask; the reference's argument checks hold."""
    from hackable_lm_b200 import kernels

    q = torch.empty(2, 64, 4, 128, device="meta", dtype=torch.bfloat16)
    for name in ("flash_attn_2", "flash_attn_3", "flash_attn_4"):
        y = kernels.scaled_dot_product_attention(q, q, q, 0.0, is_causal=True, attn_mask=None,
                                                 window_size=16, backend=name)
        assert y.shape == q.shape
        with pytest.raises(RuntimeError, match="expects window_size"):
            kernels.scaled_dot_product_attention(q, q, q, 0.0, attn_mask=torch.ones(1, device="meta"),
                                                 backend=name)
    qt = q.transpose(1, 2)
    bm = kernels.flex_attention_block_mask(2, 4, 64, torch.device("meta"), 16)
    y = kernels.scaled_dot_product_attention(qt, qt, qt, 0.0, is_causal=True, block_mask=bm,
                                             window_size=16, backend="flex_attention")
    assert y.shape == qt.shape
    with pytest.raises(RuntimeError, match="dropout"):
        kernels.scaled_dot_product_attention(qt, qt, qt, 0.1, block_mask=bm, backend="flex_attention")
    with pytest.raises(RuntimeError, match="unsupported attention backend"):
        kernels.scaled_dot_product_attention(qt, qt, qt, 0.0, backend="nope")


def test_window_mask_matches_reference_mask(reference_modules):
    """The window mask this path builds equals the reference AttentionCore's own
    (model.py:143-153) for a windowed layer."""
    ref_config, ref_model = reference_modules
    from hackable_lm_b200.config import layer_attention_window

    cfg = ref_config.resolve_config(depth=4, vocab_size=64, sequence_len=32, device_batch_size=1,
                                    attention_window=8, attention_backend="torch").model
    core = ref_model.AttentionCore(cfg, 0)
    ref_mask = core._sliding_window_mask(32, torch.device("cpu"))[0, 0]
    w = layer_attention_window(0, cfg.n_layer, cfg.attention_window, cfg.attention_full_every)
    pos = torch.arange(32)
    dist = pos[:, None] - pos[None, :]
    assert torch.equal((dist >= 0) & (dist < w), ref_mask)
