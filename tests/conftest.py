"""Test setup: the in-tree package and the oracle on sys.path, the `gpu` marker, shared fixtures.

`-m gpu` tests run the B200 kernels through the C ABI / the custom ops and compare them with the
oracle (oracle/xdna_oracle.py, pinned to the reference by tests/test_oracle.py). `-m "not gpu"`
tests need no GPU: the oracle against the golden vectors, host logic, and that libxdna_b200.so
loads and exports every symbol include/xdna_b200.h declares.
"""

import json
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "torch-xdna_b200"
for p in (str(PKG), str(ROOT), str(ROOT / "tests" / "golden")):
    if p not in sys.path:
        sys.path.insert(0, p)

LIB = PKG / "torch_xdna" / "lib" / "libxdna_b200.so"
GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU")


def ensure_built():
    """Build libxdna_b200.so in-tree if it is missing (nvcc cross-compiles without a GPU)."""
    if not LIB.exists():
        subprocess.run(["make", "-j8", "-C", str(PKG / "csrc")], check=True, capture_output=True)
    return LIB


@pytest.fixture(scope="session")
def golden():
    manifest = json.loads((GOLDEN / "golden.json").read_text())
    arrays = np.load(GOLDEN / "golden.npz")
    return manifest, arrays


@pytest.fixture(scope="session")
def cuda():
    import torch

    import torch_xdna

    if not torch_xdna.gpu_available():
        pytest.fail(f"GPU test without a usable B200: {torch_xdna.kernels.unavailable_reason()}")
    return torch.device("cuda", torch.cuda.current_device())
