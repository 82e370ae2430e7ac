import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

GOLDEN = os.path.join(REPO, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: takes more than a few seconds on a CPU")


def golden(name):
    import torch
    return torch.load(os.path.join(GOLDEN, f"{name}.pt"), weights_only=False)


@pytest.fixture(scope="session")
def a8():
    """The product package (its directory name is not a Python identifier, so it is loaded by path)."""
    from __graft_entry__ import load_package
    return load_package()


@pytest.fixture(scope="session")
def tiny_model():
    from oracle.standin import build_standin, tiny_config
    return build_standin(0, tiny_config())
