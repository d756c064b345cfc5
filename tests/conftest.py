"""Shared test setup: import paths and the ``gpu`` marker.

Tests marked ``gpu`` need a B200 and the built CUDA runtime library; every
other test runs on a CPU-only machine.
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (os.path.join(ROOT, "emmy-ptx_b200"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU and the built libemmyrt.so")
