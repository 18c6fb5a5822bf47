import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line(
        "markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")
    config.addinivalue_line("markers", "slow: long-running test")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without a CUDA device")
    return torch.device("cuda:0")


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Measured max-abs errors of the parity checks, per precision."""
    try:
        import parity
    except Exception:
        return
    lines = parity.summary_lines()
    if lines:
        terminalreporter.write_sep("-", "parity: measured max-abs error per precision")
        for line in lines:
            terminalreporter.write_line(line)
