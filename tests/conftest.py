"""Shared test set-up: repo on sys.path, the `gpu` marker, and library fixtures.

`-m "not gpu"` tests run on any machine (oracle against golden vectors, host logic,
library exports). `-m gpu` tests need a CUDA device and call the sm_100a kernels
through the C-ABI; they compare with the oracle (CPU restatement) and with the
reference's own kernels compiled for sm_100a (oracle/_ref).
"""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle

    return Oracle()


def allclose_report(got, want, atol=2e-3, rtol=1e-2):
    """|got - want| <= atol + rtol*|want| elementwise; returns (ok, max_abs, worst_index)."""
    import torch

    g = got.float().flatten().cpu()
    w = want.float().flatten().cpu()
    diff = (g - w).abs()
    bad = diff > (atol + rtol * w.abs())
    ok = not bool(bad.any()) and not bool(torch.isnan(g).any())
    idx = int(diff.argmax()) if diff.numel() else -1
    return ok, float(diff.max()) if diff.numel() else 0.0, idx
