"""Pin the CPU oracle against golden vectors produced by the reference's own CPU code."""
from __future__ import annotations

import torch

import oracle

F64 = torch.float64


def close(a, b, atol=1e-5, rtol=1e-5):
    a = torch.as_tensor(a).double()
    b = torch.as_tensor(b).double()
    assert a.shape == b.shape, (a.shape, b.shape)
    torch.testing.assert_close(a, b, atol=atol, rtol=rtol)


def c1_inputs():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(4, 256, 384, generator=g)
    residual = torch.randn(4, 256, 384, generator=g)
    weight = 1.0 + torch.randn(384, generator=g) * 0.02
    grad = torch.randn(4, 256, 384, generator=g)
    return x, residual, weight, grad


def fingerprint(t):
    flat = t.reshape(-1).double()
    return torch.stack([flat.sum(), flat.abs().sum(), flat[:8].sum(), flat[-8:].sum()])


def test_rmsnorm_c1_matches_reference(golden):
    gd = golden("rmsnorm_c1")
    x, residual, weight, grad = c1_inputs()
    for name, t in (("x", x), ("residual", residual), ("weight", weight), ("grad", grad)):
        close(fingerprint(t), gd["fingerprint"][name], atol=1e-6, rtol=0)
    out, norm = oracle.residual_rms_norm(residual, x, 1e-6, weight=weight, compute=F64)
    dx, dw = oracle.residual_rms_norm_backward(out, None, grad, 1e-6, weight=weight, compute=F64)
    rows = gd["rows"]
    flat = lambda t: t.reshape(1024, 384)[rows]  # noqa: E731
    close(flat(out), gd["out"], atol=1e-6)
    close(flat(norm), gd["norm"], atol=1e-5)
    close(flat(dx), gd["grad_x"], atol=1e-5)
    close(flat(dx), gd["grad_residual"], atol=1e-5)
    close(dw, gd["grad_weight"], atol=2e-4, rtol=1e-5)


def test_residual_rms_norm_matches_reference(golden):
    gd = golden("residual_rms_norm")
    out, norm = oracle.residual_rms_norm(gd["residual"], gd["branch"], gd["eps"], compute=F64)
    close(out, gd["out"])
    close(norm, gd["norm"])
    dx, _ = oracle.residual_rms_norm_backward(out, gd["grad_out"], gd["grad_norm"], gd["eps"], compute=F64)
    close(dx, gd["grad_residual"])
    close(dx, gd["grad_branch"])


def test_swiglu_matches_reference(golden):
    for case in golden("swiglu")["cases"]:
        close(oracle.swiglu(case["gate_up"], compute=F64), case["out"], atol=1e-6)
        close(oracle.swiglu_backward(case["gate_up"], case["grad_out"], compute=F64), case["grad_gate_up"],
              atol=1e-6)


def test_rope_tables_match_reference(golden):
    for case in golden("rope_tables")["cases"]:
        cos, sin = oracle.rope_tables(128, case["T"], case["theta"], case["fraction"])
        close(cos, case["cos"], atol=0, rtol=0)
        close(sin, case["sin"], atol=0, rtol=0)


def test_qk_norm_rope_matches_reference(golden):
    for case in golden("qk_norm_rope")["cases"]:
        qo, ko = oracle.qk_norm_rope(case["q"], case["k"], case["cos"], case["sin"], case["eps"], compute=F64)
        close(qo, case["q_out"])
        close(ko, case["k_out"])
        gq, gk = oracle.qk_norm_rope_backward(case["q"], case["k"], case["grad_q_out"], case["grad_k_out"],
                                              case["cos"], case["sin"], case["eps"], compute=F64)
        close(gq, case["grad_q"], atol=2e-5)
        close(gk, case["grad_k"], atol=2e-5)


def test_qkv_projection_matches_reference(golden):
    gd = golden("qkv")
    q, k, v = oracle.qkv_rope(gd["x"], gd["w_qkv"], gd["cos"], gd["sin"], gd["n_head"], gd["n_kv_head"],
                              gd["eps"], compute=F64)
    close(q, gd["q"], atol=2e-5)
    close(k, gd["k"], atol=2e-5)
    close(v, gd["v"], atol=2e-5)
    gx, gw = oracle.qkv_rope_backward(gd["x"], gd["w_qkv"], gd["cos"], gd["sin"], gd["grad_q_out"],
                                      gd["grad_k_out"], gd["grad_v_out"], gd["n_head"], gd["n_kv_head"],
                                      gd["eps"], compute=F64)
    close(gx, gd["grad_x"], atol=1e-4)
    close(gw, gd["grad_w"], atol=1e-4)


def test_lm_head_chunked_matches_reference(golden):
    gd = golden("lm_head")["chunked"]
    loss, gx, gw = oracle.lm_head_ce(gd["hidden"], gd["weight"], gd["targets"], gd["ignore_index"],
                                     gd["chunk"], compute=F64)
    close(loss, gd["loss"], atol=1e-6)
    close(gx.reshape(gd["grad_hidden"].shape), gd["grad_hidden"], atol=1e-6)
    close(gw, gd["grad_weight"], atol=1e-6)


def test_lm_head_ignore_index_matches_reference(golden):
    gd = golden("lm_head")["dense_ignore"]
    loss, gx, gw = oracle.lm_head_ce(gd["hidden"], gd["weight"], gd["targets"], gd["ignore_index"],
                                     0, compute=F64)
    close(loss, gd["loss"], atol=1e-6)
    close(gx, gd["grad_hidden"], atol=1e-6)
    close(gw, gd["grad_weight"], atol=1e-6)
    # ignored rows carry no gradient
    ignored = gd["targets"] == gd["ignore_index"]
    assert ignored.any()
    assert torch.count_nonzero(gx[ignored]) == 0


def test_lm_head_chunking_is_invariant():
    g = torch.Generator().manual_seed(5)
    h = torch.randn(50, 32, generator=g)
    w = torch.randn(40, 32, generator=g) * 0.1
    t = torch.randint(0, 40, (50,), generator=g)
    t[::7] = -1
    a = oracle.lm_head_ce(h, w, t, -1, 0, compute=F64)
    b = oracle.lm_head_ce(h, w, t, -1, 16, compute=F64)
    for x, y in zip(a, b):
        close(x, y, atol=1e-12, rtol=1e-12)
