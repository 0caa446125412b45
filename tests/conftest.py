"""Shared test setup.

`-m "not gpu"` runs everything that needs no GPU (oracle vs golden vectors,
host logic, the C-ABI library loading and exporting its symbols, multi-rank
sharding on gloo). `-m gpu` runs the parity tests proper: the CUDA kernels
and the layer stack through the C ABI against the CPU oracle. GPU tests skip
(not fail) on a machine without an sm_100 device.
"""
from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import torch  # noqa: E402


def _has_sm100() -> bool:
    try:
        return (torch.cuda.is_available() and torch.cuda.device_count() > 0
                and torch.cuda.get_device_capability(0)[0] == 10)
    except Exception:
        return False


HAS_GPU = _has_sm100()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    from parity_log import RECORDS
    if not RECORDS:
        return
    terminalreporter.write_sep("-", "parity against the oracle (envelope = max |err| / allowed)")
    for what, res in RECORDS:
        terminalreporter.write_line(f"{what}: {res}")


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="needs an sm_100 GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session", autouse=True)
def _no_tf32_in_references():
    """Torch-side references run in full fp32 (TF32 off) so they are exact."""
    if HAS_GPU:
        torch.backends.cuda.matmul.allow_tf32 = False
        torch.backends.cudnn.allow_tf32 = False
    yield


def tf32_round(t: torch.Tensor) -> torch.Tensor:
    """Round fp32 to the nearest TF32 value (ties away from zero), as the
    kernels' cvt.rna.tf32.f32 does: add half an ulp of the 10-bit mantissa to
    the magnitude bits and clear the 13 dropped bits."""
    bits = t.contiguous().view(torch.int32)
    rounded = (bits + 0x1000) & ~0x1FFF
    return rounded.view(torch.float32)
