"""Shared fixtures.  Tests marked ``gpu`` need a B200; the rest run on CPU."""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import __graft_entry__ as graft  # noqa: E402

GOLDEN = Path(__file__).resolve().parent / "golden"

# BASELINE tolerances: bf16 outputs rtol 2e-2 / atol 1e-2, state max-abs 1e-3.
O_RTOL, O_ATOL, S_ATOL = 2e-2, 1e-2, 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available() and torch.cuda.get_device_capability(0) == (10, 0)
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if has_gpu():
        return
    skip = pytest.mark.skip(reason="needs a B200 (sm_100) GPU")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def pkg():
    graft.build()
    return graft.package()


@pytest.fixture(scope="session")
def inputs(pkg):
    return graft.submodule("inputs")


@pytest.fixture(scope="session")
def orc():
    o = graft.oracle()
    o.build()
    return o


@pytest.fixture(scope="session")
def golden():
    def load(name):
        with np.load(GOLDEN / name) as z:
            return {k: z[k] for k in z.files}
    return load
