import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Certified near-ties of the GPU parity tests (sampled ids that differ
    from the oracle by a float32-rounding tie), with their measured gaps."""
    try:
        from tests.parity_util import CERTIFIED, TIE_ULPS
    except Exception:
        return
    tr = terminalreporter
    if not CERTIFIED:
        tr.write_line(f"parity: 0 certified near-ties (bound {TIE_ULPS} float32 ulps)")
        return
    worst = max(c[4] for c in CERTIFIED)
    kinds = {}
    for c in CERTIFIED:
        kinds[c[3]] = kinds.get(c[3], 0) + 1
    tr.write_line(f"parity: {len(CERTIFIED)} certified near-ties (bound {TIE_ULPS} float32 ulps), "
                  f"largest gap {worst:.2f}, by kind {kinds}")
    for c in CERTIFIED:
        tr.write_line(f"  {c[0]} position ({c[1]},{c[2]}) {c[3]} gap {c[4]:.2f}")
