"""CPU oracle for the hackable-lm operator hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU with PyTorch tensors, the reference
algorithm of every operator on the path (forward and backward), each function
citing the reference file:line it follows.  It is the parity checker used by
``tests/``, by ``__graft_entry__.smoke()`` and by ``bench.py`` (the
``cpu_baseline`` leg and ``--impl reference``).  The product package
``hackable_lm_b200`` never imports it and never falls back to it.

Pinning: ``tests/test_oracle_golden.py`` checks these functions against golden
vectors produced by running the reference's own CPU code
(``tests/golden/make_golden.py``).
"""
from .hotpath import (  # noqa: F401
    apply_partial_rope,
    lm_head_ce,
    qk_norm_rope,
    qk_norm_rope_backward,
    qkv_rope,
    qkv_rope_backward,
    residual_rms_norm,
    residual_rms_norm_backward,
    rms_norm,
    rope_tables,
    swiglu,
    swiglu_backward,
)
