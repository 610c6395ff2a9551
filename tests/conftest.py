"""pytest configuration: the `gpu` marker, import paths, and the in-tree builds.

`-m "not gpu"` runs the oracle checks, host logic, C-ABI load/export checks and
the gloo multi-process tests on CPU. `-m gpu` runs the parity tests proper,
which call the CUDA kernels through the C-ABI on a B200.
"""

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "tenferro-decision-rs_b200")
for path in (ROOT, PKG, os.path.dirname(os.path.abspath(__file__))):
    if path not in sys.path:
        sys.path.insert(0, path)

# libtfx.so is normally built by __graft_entry__.build(); build it here when a
# checkout runs the tests first (nvcc cross-compiles without a GPU).
if not os.path.exists(os.path.join(PKG, "lib", "libtfx.so")):
    import importlib.util

    _spec = importlib.util.spec_from_file_location("tfx_build", os.path.join(PKG, "build.py"))
    _mod = importlib.util.module_from_spec(_spec)
    _spec.loader.exec_module(_mod)
    _mod.build()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 GPU (sm_100a)")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle as orc_mod
    orc_mod.build()
    return orc_mod
