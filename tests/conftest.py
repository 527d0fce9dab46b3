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


def outside_envelope(got, runs):
    """Elements of `got` whose bytes match none of the reference runs.

    The reference head-RMSNorm sums squares with a shared-memory atomicAdd
    (src/kernels.cu:103). Measured on B200, the order of those adds changes from run
    to run (about six distinct fp32 sums per head over 25 runs), which in rare
    elements moves the 16-bit result by one unit. A value matches the reference when
    it equals the reference's result in at least one run."""
    import torch

    g = got.view(torch.int16).flatten()
    ok = torch.zeros_like(g, dtype=torch.bool)
    for r in runs:
        ok |= g == r.view(torch.int16).flatten()
    return int((~ok).sum().item())


def assert_in_reference_envelope(got, runs, max_fraction=1e-4):
    """`got` equals a reference result in every element, except at most a fraction
    `max_fraction` of elements, each within one 16-bit unit (same sign) of a value the
    reference produced: the reference's own run-to-run variation, which a finite
    number of reference runs does not always exhibit."""
    import torch

    g = got.view(torch.int16).flatten().to(torch.int32)
    R = torch.stack([r.view(torch.int16).flatten().to(torch.int32) for r in runs])
    exact = (R == g).any(0)
    near = ((R - g).abs() <= 1).any(0)
    n_out = int((~exact).sum().item())
    assert bool(near.all()), f"{int((~near).sum())} elements more than one unit from every reference run"
    assert n_out <= max(1, int(g.numel() * max_fraction)), f"{n_out} of {g.numel()} elements outside the envelope"
    return n_out
