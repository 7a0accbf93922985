"""Shared pytest configuration: the ``gpu`` marker and import paths."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and the built library")


def pytest_sessionfinish(session, exitstatus):
    """With FNA2_PARITY_REPORT set, write every parity check's errors and
    bound (tests/parity.py REPORT) there as JSON lines."""
    path = os.environ.get("FNA2_PARITY_REPORT")
    if not path:
        return
    try:
        from tests import parity
    except Exception:
        return
    import json
    with open(path, "w") as f:
        for r in parity.REPORT:
            f.write(json.dumps(r) + "\n")
