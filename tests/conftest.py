import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.pt")
REF_GOLDEN = os.path.join(ROOT, "tests", "golden", "reference_golden.pt")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: large shapes, minutes of CPU oracle time")


def pytest_collection_modifyitems(config, items):
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def golden():
    return torch.load(GOLDEN, weights_only=False)


@pytest.fixture(scope="session")
def ref_golden():
    """Outputs of the reference's own CutileGPT.forward / generate (tests/golden/make_reference_golden.py)."""
    return torch.load(REF_GOLDEN, weights_only=False)
