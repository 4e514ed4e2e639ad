import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "burn-extended_b200"), os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


def pytest_collection_modifyitems(config, items):
    if gpu_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    try:
        from moe_testutil import MAX_ABS_TOL, MARGINS, REL_L2_TOL
    except Exception:
        return
    if not MARGINS:
        return
    tr = terminalreporter
    tr.write_sep("-", f"layer output margins (bounds: max_abs {MAX_ABS_TOL:g}, rel_l2 {REL_L2_TOL:g})")
    for tag, max_abs, rel in MARGINS:
        tr.write_line(f"{tag:<60s} max_abs {max_abs:.3e}  rel_l2 {rel:.3e}")
