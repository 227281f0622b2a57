"""pytest configuration.

Mirrors the reference harness's options and fixture names
(tests/conftest.py:10-45, tests/components/test_*.py fixtures): the module
fixtures return a :class:`frank_b200.B200Module`, whose methods take numpy
arrays and return numpy arrays like the IREE modules did.  Tests that need a
B200 are marked ``gpu``.
"""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "frank-models_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

GOLDEN = REPO / "tests" / "golden"


def pytest_addoption(parser):
    parser.addoption("--backend", action="store", default="b200",
                     help="backend for the component fixtures (only 'b200' exists here)")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")
    config.addinivalue_line("markers", "slow: large-size GPU case")


@pytest.fixture(scope="session")
def backend(request):
    b = request.config.getoption("--backend")
    if b != "b200":
        pytest.skip(f"backend {b!r} is not available in this build")
    return b


@pytest.fixture(scope="session")
def b200_module(backend):
    import torch

    if not torch.cuda.is_available():
        pytest.fail("gpu test selected but no CUDA device is visible")
    from frank_b200 import B200Module

    return B200Module()


@pytest.fixture(scope="session")
def mul_mat_id_module(b200_module):
    return b200_module


@pytest.fixture(scope="session")
def moe_ffn_module(b200_module):
    return b200_module


@pytest.fixture(scope="session")
def swiglu_module(b200_module):
    return b200_module
