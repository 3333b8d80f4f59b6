"""Shared pytest setup.

Markers: `gpu` tests need a CUDA device (run on the B200 box); everything else
runs on CPU.  The product binding (voxtral.cpp_b200/vxk.py) and the oracle
binding (oracle/vx_oracle.py) are put on sys.path here; tests are the only
code besides smoke() and bench.py that may import the oracle.
"""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
for sub in ("voxtral.cpp_b200", "oracle"):
    p = str(ROOT / sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


@pytest.fixture(scope="session")
def vxk():
    import vxk as mod

    mod.load()
    return mod


@pytest.fixture(scope="session")
def oracle():
    import vx_oracle as mod

    mod.lib()
    return mod
