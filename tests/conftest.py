"""Shared fixtures for the pulsar_b200 test-suite.

Markers: ``gpu`` (needs a CUDA device; run on the B200 box) and ``slow``. The CPU suite
(``-m "not gpu"``) checks the oracle against the reference's golden vectors, the host
logic and the C-ABI library's symbol table.
"""

from __future__ import annotations

import math
import os
import sys

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "pulsar-300m_b200")
for p in (PKG, REPO):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(REPO, "tests", "golden")
HAS_CUDA = torch.cuda.is_available()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: requires a CUDA device (B200)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds")


def load_golden(name: str):
    path = os.path.join(GOLDEN, f"{name}.pt")
    if not os.path.exists(path):
        pytest.skip(f"golden fixture {name}.pt not generated")
    return torch.load(path, weights_only=False)


def assert_close(actual, expected, *, atol=2e-2, rtol=2e-2, msg=""):
    """Fails only when BOTH max-abs > atol and max-rel > rtol (the reference's rule,
    tests/conftest.py:118-144 of the reference)."""
    a = actual.detach().float().cpu()
    e = expected.detach().float().cpu()
    if a.shape != e.shape:
        raise AssertionError(f"{msg}: shape mismatch {tuple(a.shape)} vs {tuple(e.shape)}")
    max_abs = (a - e).abs().max().item() if a.numel() else 0.0
    max_rel = ((a - e).abs() / e.abs().clamp_min(1e-6)).max().item() if a.numel() else 0.0
    if not (math.isfinite(max_abs) and math.isfinite(max_rel)):
        raise AssertionError(f"{msg}: non-finite values (max_abs={max_abs}, max_rel={max_rel})")
    if max_abs > atol and max_rel > rtol:
        raise AssertionError(f"{msg}: max_abs={max_abs:.3e} (atol {atol:.1e}), max_rel={max_rel:.3e} (rtol {rtol:.1e})")


@pytest.fixture
def gpu():
    if not HAS_CUDA:
        pytest.skip("CUDA not available")
    return torch.device("cuda")
