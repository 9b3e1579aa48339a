"""Shared fixtures. GPU tests carry @pytest.mark.gpu; everything else runs on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
GOLDEN = ROOT / "tests" / "golden"
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def oracle():
    from oracle.pyoracle import Oracle

    return Oracle()


@pytest.fixture(scope="session")
def ref():
    from oracle.pyoracle import REF_LIB, Reference

    if not REF_LIB.exists():
        pytest.skip("reference build oracle/_ref is absent")
    return Reference()


@pytest.fixture(scope="session")
def kb():
    import kadan_b200

    return kadan_b200


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test needs a CUDA device")
    return torch.device("cuda:0")


def rel_err(got, want) -> float:
    """max|got - want| / max(max|want|, 1): the reference's own GEMV check
    (IW/tests/gguf_text.cpp:247-250)."""
    import numpy as np

    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    return float(np.max(np.abs(got - want)) / max(float(np.max(np.abs(want))), 1.0))
