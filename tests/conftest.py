import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))
if str(ROOT / "tests") not in sys.path:
    sys.path.insert(0, str(ROOT / "tests"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    import oracle

    return oracle.load("port")


@pytest.fixture(scope="session")
def orc_ref():
    import oracle

    if not oracle.has_ref():
        pytest.skip("oracle/_ref not built (reference sources absent)")
    return oracle.load("ref")


def pytest_sessionfinish(session, exitstatus):
    """With YATTN_PARITY_LOG set, writes every parity check's error and floor
    (oracle.PARITY_LOG) there as JSON."""
    import json
    import os

    path = os.environ.get("YATTN_PARITY_LOG")
    if not path:
        return
    import oracle

    with open(path, "w") as f:
        json.dump(oracle.PARITY_LOG, f, indent=0)
