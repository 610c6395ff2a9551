"""pytest configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs the oracle checks, host logic, C-ABI load/export checks and
the gloo multi-process tests on CPU. `-m gpu` runs the parity tests proper,
which call the CUDA kernels through the C-ABI on a B200.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tenferro-decision-rs_b200")
for path in (ROOT, PKG):
    if path not in sys.path:
        sys.path.insert(0, path)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as orc_mod
    orc_mod.build()
    return orc_mod
