import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session", autouse=True)
def _built():
    """Builds the CUDA library (cross-compiles without a GPU) and the CPU oracle once."""
    from hybridagent_b200 import build as hb
    from oracle import zero1
    hb.build()
    zero1.build()
