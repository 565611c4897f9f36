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


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Tally of which parity criterion each kernel-vs-fp32 comparison passed
    (tests/helpers.py::assert_close: A = north-star bound, A0 = max-abs against
    a ~zero reference, B = plus storage rounding, C = against the
    rounding-emulated fp32 math, D = within the first-order rounding bound)."""
    try:
        from helpers import REPORT
    except ImportError:
        return
    if not REPORT:
        return
    counts = {}
    for _, crit, _, _ in REPORT:
        counts[crit] = counts.get(crit, 0) + 1
    # cosine is not meaningful against a ~zero reference (criterion A0)
    worst_cos = min((c for _, crit, _, c in REPORT if crit != "A0"), default=1.0)
    tally = ", ".join(f"{k}={counts[k]}" for k in sorted(counts))
    for name, crit, m, c in REPORT:
        if crit in ("B", "C", "D"):
            terminalreporter.write_line(f"  parity {crit}: {name} max_abs={m:.3e} cos={c:.7f}")
    terminalreporter.write_line(f"parity criteria: {len(REPORT)} comparisons: {tally}; lowest cosine (A-D) {worst_cos:.7f}")
