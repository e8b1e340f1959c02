"""Shared pytest configuration: the `gpu` marker and import paths."""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in (ROOT, os.path.join(ROOT, "x-minimaxh3_b200")):
    if sub not in sys.path:
        sys.path.insert(0, sub)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")
