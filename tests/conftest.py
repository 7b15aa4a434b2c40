import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built libsvla.so")


@pytest.fixture(scope="session")
def golden():
    import json
    return json.loads((REPO / "tests" / "golden" / "golden.json").read_text())


@pytest.fixture(scope="session")
def golden_dir():
    return REPO / "tests" / "golden"
