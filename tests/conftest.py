import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def _keep_freed_heap_memory():
    """Let glibc keep freed large blocks in the heap instead of returning them
    to the OS: the CPU oracle allocates many large temporaries in a row, and
    faulting fresh pages in for each one dominated its run time."""
    try:
        import ctypes

        libc = ctypes.CDLL("libc.so.6")
        libc.mallopt(-3, 32 << 20)  # M_MMAP_THRESHOLD: the largest value glibc accepts on 64-bit
        libc.mallopt(-1, 1 << 30)   # M_TRIM_THRESHOLD
    except OSError:
        pass


_keep_freed_heap_memory()

# Parity tolerance of the north star: fp32 outputs and gradients within
# 1e-5 relative / 1e-6 absolute of the reference.
RTOL = 1e-5
ATOL = 1e-6


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (B200, sm_100a) device")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container (run with -m gpu on a B200)")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_sessionfinish(session, exitstatus):
    """Write the per-tensor parity figures gathered by tests/parity.py to the
    JSON file named by VMSCAN_PARITY_TABLE (unset: nothing is written)."""
    path = os.environ.get("VMSCAN_PARITY_TABLE")
    if not path:
        return
    import json

    from parity import RECORDS

    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "w") as f:
        json.dump(RECORDS, f, indent=0)
