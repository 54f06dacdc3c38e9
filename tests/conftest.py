"""Test configuration: import paths, the ``gpu`` marker and shared helpers."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
PKG_ROOT = ROOT / "robotics-batch-invariant-ops_b200"
for p in (str(PKG_ROOT), str(ROOT)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="CUDA device required")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


# Tolerances of the reference suite (test_batch_invariance.py:28-32).
TOLERANCES = {
    torch.float32: {"rtol": 5e-5, "atol": 2e-5},
    torch.float16: {"rtol": 2e-3, "atol": 1e-3},
    torch.bfloat16: {"rtol": 2e-2, "atol": 1e-2},
}
DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def assert_first_sample_equal(alone: torch.Tensor, batched: torch.Tensor) -> None:
    """Bitwise B=1 vs slice-of-B=N check (reference test_batch_invariance.py:35-39)."""
    assert torch.equal(alone, batched[:1]), (
        f"first sample changed: max diff "
        f"{(alone.float() - batched[:1].float()).abs().max().item()}"
    )


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """Every GPU test must leave the library's device status word clear (no
    bounded wait timed out, no index check fired)."""
    if "gpu" not in request.keywords or not torch.cuda.is_available():
        yield
        return
    from batch_invariant_ops import _lib

    _lib.clear_device_status()
    yield
    status = _lib.device_status()
    assert status == 0, f"device status word set: {status:#x}"
