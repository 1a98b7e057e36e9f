"""Shared fixtures.  `-m gpu` tests need a CUDA device (a B200); everything
else runs on the CPU.  The CPU oracle (oracle/) is the parity checker; the
reference's own kernels (oracle/_ref/omo_ref*.so, built from the reference
sources by oracle/build_ref.py) are a second checker when present."""
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "mxfp4-hopper_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: full-size workloads")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def ref_kernels():
    """The reference's kernels compiled from its sources, or skip."""
    import importlib
    d = ROOT / "oracle" / "_ref"
    if not any(d.glob("omo_ref*.so")):
        pytest.skip("oracle/_ref not built")
    if str(d) not in sys.path:
        sys.path.insert(0, str(d))
    return importlib.import_module("omo_ref")
