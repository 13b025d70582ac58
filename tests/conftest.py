import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


import json

import pytest

_REPORT = {}


@pytest.fixture
def parity_report():
    """Per-case parity figures (kept positions that differ from the reference, score
    errors); written as JSON to $CKV_PARITY_REPORT at the end of the session."""
    return _REPORT


def pytest_sessionfinish(session, exitstatus):
    path = os.environ.get("CKV_PARITY_REPORT")
    if path and _REPORT:
        with open(path, "w") as f:
            json.dump(_REPORT, f, indent=1, sort_keys=True)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200); runs the sm_100a kernels")
