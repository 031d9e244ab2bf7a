import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_terminal_summary(terminalreporter):
    helpers = sys.modules.get("tests.helpers")
    if helpers is None or not helpers.PARITY:
        return
    terminalreporter.write_sep("-", "attention parity against the oracle (worst per case)")
    for name, (mx, rms, rows) in sorted(helpers.PARITY.items()):
        terminalreporter.write_line(f"{name:48s} max-abs {mx:.3e}  rms {rms:.3e}  rows {rows}")


@pytest.fixture(scope="session")
def golden():
    import numpy as np
    return np.load(ROOT / "tests" / "golden" / "numpyqwen_t40.npz")


@pytest.fixture(scope="session")
def golden200():
    import numpy as np
    return np.load(ROOT / "tests" / "golden" / "numpyqwen_t200.npz")
