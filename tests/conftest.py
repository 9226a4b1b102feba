import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _has_cuda() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if _has_cuda():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def _reference_root():
    """A yz29528/tokenFactory checkout for the tests that compare against the reference's own
    classes: $TOKENFACTORY_REFERENCE, else a `reference` directory next to this repository."""
    for cand in (os.environ.get("TOKENFACTORY_REFERENCE"),
                 os.path.join(os.path.dirname(ROOT), "reference")):
        if cand and os.path.isdir(os.path.join(cand, "qwen3_8")):
            return cand
    return None


@pytest.fixture(scope="session")
def reference_root():
    root = _reference_root()
    if root is None:
        pytest.skip("reference checkout not available")
    if root not in sys.path:
        sys.path.insert(0, root)
    return root
