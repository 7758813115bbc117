"""The B200 model against the reference's own LanguageModel (BASELINE config 5's model
and a windowed depth-4 model), through the golden fixtures that
tests/golden/make_golden.py made by running the reference model on the CPU in fp32.

The weights are re-created from the fixture's seed by this package's model (same
init order as the reference; the stored init fingerprints are checked), rounded to
bf16 as the training precision policy does, and one forward + backward runs on the
B200 operators.  The bars:

* loss within 1e-3 relative of the reference's (fp32) loss;
* every parameter's gradient norm within 1e-2 relative;
* the stored gradient rows (a few seeded rows per parameter) of every parameter
  within 2x (+1e-2) the relative L2 error of the reference's own formulation run in
  bf16 on the same GPU (this package's "torch" backend, pinned to the reference
  model at 1e-5 by tests/test_model_cpu.py), and, averaged over the parameters, no
  further from the fp32 reference than that bf16 run.  Per parameter the sampled
  rows are noisy: the bf16 reference formulation itself ranges from 0.8e-2 to
  7e-2 over the d12 parameters.  Whole-model gradients through many bf16
  layers do not meet an elementwise 2e-2 bar even when computed by the reference
  itself in bf16 (measured: max|err|/rms 0.04-0.12 at depth 4), so the
  per-element metric is recorded for every parameter (HLM_PARITY_LOG) and the
  bar is set by the reference's own bf16 execution.
"""
from __future__ import annotations

import pytest
import torch

import model_golden as mg
from parity import assert_loss_close, record

pytestmark = pytest.mark.gpu


def _run(gd, backend, device, attention_backend=None):
    from hackable_lm_b200 import kernels

    model = mg.build(gd, backend, attention_backend).to(device)
    kernels.apply_precision_policy(model, "bf16")
    x, y = mg.batch(gd, device)
    _, loss = model(x, y)
    loss.backward()
    torch.cuda.synchronize()
    return model, loss.detach().double().item()


def _row_rel_l2(model, gd):
    out = {}
    for n, p in model.named_parameters():
        rows, ref = gd["grad_rows"][n]
        got = p.grad.detach().double().cpu()[rows]
        ref = ref.double()
        out[n] = ((got - ref).norm() / ref.norm()).item(), ((got - ref).abs().max() / ref.pow(2).mean().sqrt()).item()
    return out


@pytest.mark.parametrize("attention", ["sdpa", "b200"])
@pytest.mark.parametrize("name", ["model_d4_window", "model_d12"])
def test_b200_model_matches_reference_model(name, attention, golden, cuda_device):
    """With the attention core on SDPA (the default) and on this library's tcgen05
    forward (attention_backend "b200": sliding windows in three of the d4 model's
    four layers); the latter also checks that the forward kernel ran in every layer."""
    from hackable_lm_b200 import _lib

    from hackable_lm_b200.config import layer_attention_window

    gd = golden(name)
    _lib.clear_device_error()
    c = gd["config"]
    depth = c["depth"]
    # with "sdpa" the sliding-window layers still run the tcgen05 forward (SDPA has no
    # sliding-window kernel); the full-attention layers run SDPA
    windowed = sum(1 for i in range(depth)
                   if (w := layer_attention_window(i, depth, c["window"], c["attention_full_every"])) is not None
                   and w < c["seq"])
    with _lib.KernelTimer("attn_fwd", 4 * depth) as timer:
        mb, loss_b = _run(gd, "b200", cuda_device, attention)
    assert _lib.device_error() == 0
    assert timer.launches == (depth if attention == "b200" else windowed), timer.launches
    assert_loss_close(loss_b, gd["loss"].item(), what=f"{name} loss")
    norms = mg.grad_errors(mb, gd)
    rows_b = _row_rel_l2(mb, gd)
    del mb
    mt, loss_t = _run(gd, "torch", cuda_device)
    rows_t = _row_rel_l2(mt, gd)
    del mt
    record(f"{name} loss (reference formulation in bf16)", loss_rel_err=abs(loss_t - gd["loss"].item()) / gd["loss"].item())
    bad = []
    for n, (norm_err, _) in norms.items():
        rel_b, strict_b = rows_b[n]
        rel_t, strict_t = rows_t[n]
        record(f"{name} grad {n}", norm_rel_err=norm_err, rows_rel_l2=rel_b, max_err_over_rms=strict_b,
               torch_bf16_rows_rel_l2=rel_t, torch_bf16_max_err_over_rms=strict_t)
        if norm_err > 1e-2 or rel_b > 2.0 * rel_t + 1e-2:
            bad.append((n, norm_err, rel_b, rel_t))
    assert not bad, f"gradients beyond the bar (name, norm err, rows rel L2, torch-bf16 rows rel L2): {bad}"
    mean_b = sum(r[0] for r in rows_b.values()) / len(rows_b)
    mean_t = sum(r[0] for r in rows_t.values()) / len(rows_t)
    record(f"{name} mean rows rel L2", b200=mean_b, torch_bf16=mean_t)
    assert mean_b <= mean_t, f"mean gradient-row error {mean_b:.4f} above the bf16 reference formulation's {mean_t:.4f}"


def test_b200_model_is_causal(cuda_device):
    """Changing token t+1 leaves every hidden state at positions <= t bit-identical
    (the final normed hidden state feeding the LM head), and changes position t+1."""
    from hackable_lm_b200 import config as hcfg
    from hackable_lm_b200 import kernels
    from hackable_lm_b200.model import LanguageModel

    torch.manual_seed(0)
    cfg = hcfg.model_config_for_depth(4, vocab_size=4096, sequence_len=512, attention_window=128, backend="b200")
    m = LanguageModel(cfg).to(cuda_device)
    kernels.apply_precision_policy(m, "bf16")

    def hidden(idx):
        with torch.no_grad():
            x = m.tok_emb(idx)
            xn = m.input_norm(x)
            for blk in m.blocks:
                x, xn = blk(x, xn)
        return xn

    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, 4096, (2, 512), generator=g).to(cuda_device)
    base = hidden(ids)
    for t in (0, 127, 300, 510):
        pert = ids.clone()
        pert[:, t + 1] = (pert[:, t + 1] + 17) % 4096
        h = hidden(pert)
        assert torch.equal(h[:, : t + 1], base[:, : t + 1]), f"positions <= {t} changed"
        assert not torch.equal(h[:, t + 1], base[:, t + 1])
