"""Shared fixtures.  Tests marked `gpu` need a B200 (run with -m gpu); all
others run on CPU.  The CPU oracle (oracle/) is the checker everywhere."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

import __graft_entry__ as ge  # noqa: E402


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def pkg():
    return ge.load_package()


@pytest.fixture(scope="session")
def orc():
    return ge.load_oracle()


@pytest.fixture(scope="session")
def mine(orc):
    return orc.Harness("mine")


@pytest.fixture(scope="session")
def ref(orc):
    """The caller harness built against the reference's own sources; skipped
    where oracle/_ref was not built (the golden fixtures still apply)."""
    try:
        return orc.Harness("ref")
    except OSError as e:
        pytest.skip(str(e))


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "golden.json")) as f:
        return json.load(f)


@pytest.fixture(scope="session")
def cuda():
    import torch
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    torch.cuda.set_device(0)
    return torch.device("cuda:0")
