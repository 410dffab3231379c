import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (REPO, os.path.join(REPO, "constraintflow-gpu_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")
    config.addinivalue_line("markers", "slow: long CPU case, run with CF_SLOW=1")


def pytest_collection_modifyitems(config, items):
    if os.environ.get("CF_SLOW") == "1":
        return
    skip = pytest.mark.skip(reason="slow CPU case; set CF_SLOW=1")
    for it in items:
        if "slow" in it.keywords:
            it.add_marker(skip)


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Worst observed parity ratios (error / tolerance) of this session, per case and check."""
    try:
        import parity
    except Exception:
        return
    if not parity.OBSERVED:
        return
    parity.dump_observed()
    tr = terminalreporter
    tr.section("parity: worst observed error / tolerance")
    for key in sorted(parity.OBSERVED):
        tr.write_line(f"{parity.OBSERVED[key]:10.4f}  {key}")
