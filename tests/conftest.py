import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a) and the built extension")
    config.addinivalue_line("markers", "multigpu: needs 2+ GPUs")
    config.addinivalue_line("markers", "slow: long-running CPU test")


def pytest_collection_modifyitems(config, items):
    has_gpu = torch.cuda.is_available()
    skip_gpu = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords and not has_gpu:
            it.add_marker(skip_gpu)


@pytest.fixture(autouse=True)
def _seed():
    torch.manual_seed(0)
    yield


@pytest.fixture(autouse=True)
def _symm_canaries(request):
    """After a GPU test, no symmetric buffer may have been written past its end
    (each one carries a guard tail; :mod:`bwn.parallel.symm`)."""
    yield
    mod = sys.modules.get("bwn.parallel.symm")
    if mod is not None and "gpu" in request.keywords and torch.cuda.is_available():
        bad = mod.check_canaries()
        assert not bad, f"symmetric buffers written past their end: {bad}"
