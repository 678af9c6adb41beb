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


@pytest.fixture(autouse=True)
def _name_comparisons(request):
    """Labels the comparisons a test records with the test's id."""
    import helpers

    helpers.set_current_test(request.node.nodeid.split("::")[-1])
    yield


def pytest_terminal_summary(terminalreporter):
    """The worst error of every gradient and absolute comparison of the session, per test."""
    try:
        import helpers
    except ImportError:  # pragma: no cover
        return
    if helpers.GRAD_REPORT:
        terminalreporter.write_sep("-", "gradients: worst |got - want| / max|want| (bound 1e-4)")
        worst = max(r[1] for r in helpers.GRAD_REPORT)
        for label, err, size in helpers.GRAD_REPORT:
            terminalreporter.write_line(f"{err:.3e}  {label} ({size} entries)")
        terminalreporter.write_line(f"worst over {len(helpers.GRAD_REPORT)} gradient comparisons: {worst:.3e}")
    if helpers.ABS_REPORT:
        terminalreporter.write_sep("-", "absolute comparisons: worst |got - want| (bound)")
        for label, err, atol in helpers.ABS_REPORT:
            terminalreporter.write_line(f"{err:.3e}  (bound {atol:g})  {label}")
