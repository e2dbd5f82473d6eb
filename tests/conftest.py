import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (CUDA device) to run")


def pytest_collection_modifyitems(config, items):
    """GPU tests fail loudly when asked for and no device exists; they are
    only deselected by the ``-m "not gpu"`` expression, never skipped."""
    return


@pytest.fixture(scope="session")
def rng():
    import numpy as np

    return np.random.default_rng(1234)
