import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def model_root(tmp_path_factory):
    """Synthetic models are written once per session (deterministic, seeded)."""
    root = os.environ.get("FFWD_B200_TEST_MODEL_ROOT")
    if root:
        os.makedirs(root, exist_ok=True)
        return root
    return str(tmp_path_factory.mktemp("models"))
