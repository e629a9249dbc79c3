"""Test setup: import paths, the `gpu` marker, shared helpers.

CPU tests (-m "not gpu") check the oracle against the golden fixtures, the
host-side logic, and that libnvattn.so loads and exports its C ABI. GPU tests
(-m gpu) are the parity tests proper: they call the kernels through the C ABI
and compare with the oracle on the same seeded inputs.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
PROJECT = REPO / "nano-vllm-x_b200"
GOLDEN = REPO / "tests" / "golden"
for p in (str(REPO), str(PROJECT), str(GOLDEN)):
    if p not in sys.path:
        sys.path.insert(0, p)
# The reference engine, when installed next to the repo (pip --target
# baseline/_ref), for the tests that drive nvattn from inside it.
REF_INSTALL = REPO / "baseline" / "_ref"
if REF_INSTALL.is_dir() and str(REF_INSTALL) not in sys.path:
    sys.path.append(str(REF_INSTALL))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200) device and libnvattn.so")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this environment")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def bf16_bits(t: torch.Tensor):
    """Raw 16-bit patterns of a bf16 tensor as a numpy uint16 array."""
    return t.contiguous().view(torch.int16).cpu().numpy().view("uint16")


def from_bits(a) -> torch.Tensor:
    return torch.from_numpy(a.view("int16").copy()).view(torch.bfloat16)
