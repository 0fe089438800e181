import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU and libbigrig_b200.so")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a GPU test ran without a CUDA device")
    return torch.device("cuda", 0)


def pytest_terminal_summary(terminalreporter):
    """Every exceedance count a parity test recorded (elements past the expert-output bar
    |got - want| <= 2e-3 + 1e-2 |want|), one line per comparison."""
    from tests._experts import EXCEEDANCE_REPORT
    if not EXCEEDANCE_REPORT:
        return
    terminalreporter.section("parity bar exceedance (elements outside 1e-2 rel / 2e-3 abs)")
    for test, what, r in EXCEEDANCE_REPORT:
        terminalreporter.write_line(
            f"{test}: {what}: {r['outside']} of {r['of']} outside, max |d| {r['max_abs']:.3g}, "
            f"worst {r['max_ratio']:.3g}x the bar")
