import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "gemma-triton-flash-attn_b200")
for p in (ROOT, PKG_DIR):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_sessionfinish(session, exitstatus):
    path = os.environ.get("GQAFA_PARITY_REPORT")
    if not path:
        return
    import json

    from helpers import REPORT

    with open(path, "w") as f:
        json.dump([dict(name=n, criterion=c, max_abs=m, cos=k) for n, c, m, k in REPORT], f, indent=1)
