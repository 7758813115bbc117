"""Host-side logic that runs without a GPU: configuration arithmetic, backend
resolution, the no-CPU-fallback guard, and the fake (meta) implementations the
custom operators expose to torch.compile."""
from __future__ import annotations

import pytest
import torch

from hackable_lm_b200 import config, kernels, ops


def test_d12_dimensions_and_flops():
    cfg = config.model_config_for_depth(12)
    assert (cfg.n_embd, cfg.n_head, cfg.mlp_hidden, cfg.head_dim) == (768, 6, 2048, 128)
    sp = config.scaling_params_for_depth(12, 32768)
    assert sp == 110_100_480
    assert config.estimate_flops_per_token(12, 768, 2048, sp) == 887_095_296
    assert config.estimate_flops_per_token(12, 768, 2048, sp, 512, 4) == 759_693_312


def test_gradient_accumulation_rules():
    assert config.gradient_accumulation(2**20, 16, 2048, 1) == 32
    assert config.gradient_accumulation(2**20, 16, 2048, 8) == 4
    with pytest.raises(RuntimeError):
        config.gradient_accumulation(2**20, 16, 2048, 3)
    with pytest.raises(RuntimeError):
        config.gradient_accumulation(16 * 2048, 16, 2048, 2)


def test_backend_names_and_triton_alias():
    assert config.normalize_module_backend("qkv_backend", "triton") == "b200"
    assert config.normalize_module_backend("qkv_backend", "TORCH") == "torch"
    with pytest.raises(ValueError):
        config.normalize_module_backend("qkv_backend", "cuda")
    info = kernels.resolve_kernel_backends("torch", "fp32_test", False, allow_torch_backend=True,
                                           **{f: "torch" for f in config.MODULE_BACKEND_FIELDS})
    assert all(getattr(info, f) == "torch" for f in config.MODULE_BACKEND_FIELDS)
    with pytest.raises(ValueError):
        kernels.resolve_kernel_backends("triton", "bf16", False)
    with pytest.raises(ValueError):
        kernels.resolve_kernel_backends("torch", "bf16", False, bogus_backend="torch")


def test_cpu_tensors_are_rejected_not_silently_computed():
    x = torch.randn(4, 8)
    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.swiglu_triton(x)
    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.rms_norm(x, None, 1e-6)
    with pytest.raises(RuntimeError, match="CUDA"):
        kernels.qk_norm_rope_triton(torch.randn(1, 2, 1, 8), torch.randn(1, 2, 1, 8),
                                    torch.randn(1, 2, 1, 4), torch.randn(1, 2, 1, 4), 1e-6)
    with pytest.raises(RuntimeError):
        kernels.fused_linear_cross_entropy_with_weight(x, torch.randn(16, 8), None,
                                                       torch.zeros(4, dtype=torch.long), "b200")
    with pytest.raises(RuntimeError, match="even"):
        kernels.swiglu_triton(torch.randn(4, 7))
    with pytest.raises(RuntimeError, match="backend"):
        kernels.fused_linear_cross_entropy_with_weight(x, torch.randn(16, 8), None,
                                                       torch.zeros(4, dtype=torch.long), "torch")


def test_fake_implementations_shapes():
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        gu = torch.empty(4, 16, 2 * 2048, dtype=torch.bfloat16, device="cuda")
        assert ops.swiglu(gu).shape == (4, 16, 2048)
        x = torch.empty(2, 64, 768, dtype=torch.bfloat16, device="cuda")
        w = torch.empty(2304, 768, dtype=torch.bfloat16, device="cuda")
        cos = torch.empty(1, 1, 64, 32, dtype=torch.bfloat16, device="cuda")
        q, k, v, rstd = ops.qkv_rope(x, w, cos, cos, 6, 6, 1e-6)
        assert q.shape == (2, 64, 6, 128) and v.shape == (2, 64, 6, 128) and rstd.shape == (128, 12)
        h = torch.empty(128, 768, dtype=torch.bfloat16, device="cuda")
        W = torch.empty(32768, 768, dtype=torch.bfloat16, device="cuda")
        t = torch.empty(128, dtype=torch.long, device="cuda")
        loss, gx, gw = ops.lm_head_ce(h, W, t, -1, 0, True, True)
        assert loss.shape == () and gx.shape == h.shape and gw.shape == W.shape
        out, norm = ops.residual_rms_norm(x, x, None, 1e-6)
        assert out.shape == norm.shape == x.shape


def test_attention_backward_selection():
    """The backward attention_backward runs: the tcgen05 kernel for a sliding window
    shorter than the sequence with equal q / kv heads, the library backward for full
    causal attention and grouped heads; ATTENTION_BWD overrides (never to the native
    kernel for grouped heads, which it does not handle)."""
    sel = ops._native_attention_bwd
    old = ops.ATTENTION_BWD["mode"]
    try:
        ops.ATTENTION_BWD["mode"] = "auto"
        assert sel(512, 2048, 6, 6) and sel(1, 128, 2, 2)
        assert not sel(0, 2048, 6, 6) and not sel(2048, 2048, 6, 6) and not sel(4096, 2048, 6, 6)
        assert not sel(512, 2048, 6, 2)
        ops.ATTENTION_BWD["mode"] = "native"
        assert sel(0, 2048, 6, 6) and not sel(512, 2048, 6, 3)
        ops.ATTENTION_BWD["mode"] = "library"
        assert not sel(512, 2048, 6, 6)
    finally:
        ops.ATTENTION_BWD["mode"] = old
