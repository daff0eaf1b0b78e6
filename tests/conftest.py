"""Shared pytest setup: import paths and the `gpu` marker.

`-m "not gpu"` runs everywhere (oracle vs golden vectors, host logic, the C-ABI
library's exports); `-m gpu` needs a B200 and exercises the CUDA kernels through the
C ABI.
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "pto-fuser_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (sm_100a)")
