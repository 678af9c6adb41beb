import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(REPO / "high-dimensional-splatting_b200"))
sys.path.insert(0, str(REPO / "oracle"))
sys.path.insert(0, str(REPO))

try:
    from hypothesis import settings

    settings.register_profile("dev", max_examples=8, deadline=None)
    settings.register_profile("full", max_examples=100, deadline=None)
    settings.load_profile(os.environ.get("HYPOTHESIS_PROFILE", "dev"))
except ImportError:  # pragma: no cover
    pass


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libhds_b200.so")


GOLDEN = REPO / "tests" / "golden"


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    def load(name):
        return dict(np.load(GOLDEN / name, allow_pickle=False))

    return load
