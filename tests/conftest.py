from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and the built CUDA library")


@pytest.fixture(scope="session")
def golden():
    import torch

    cache = {}

    def load(name: str):
        if name not in cache:
            cache[name] = torch.load(GOLDEN / f"{name}.pt", weights_only=False)
        return cache[name]

    return load


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test selected but CUDA is not available")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"these kernels are built for sm_100a; device is sm_{major}{minor}")
    from hackable_lm_b200 import _lib

    _lib.load()
    return torch.device("cuda", 0)


def reference_checkout():
    """A hackable-lm checkout: $HACKABLE_LM_REFERENCE, else a directory named
    ``reference`` or ``hackable-lm`` beside this repository; None without one.
    Only CPU tests read it (the GPU tests use the committed golden fixtures)."""
    import os

    cands = [os.environ.get("HACKABLE_LM_REFERENCE")] + [str(ROOT.parent / n) for n in ("reference", "hackable-lm")]
    for c in cands:
        if c and (Path(c) / "model.py").is_file() and (Path(c) / "kernels.py").is_file():
            return Path(c)
    return None
