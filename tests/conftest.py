"""Test configuration: the `gpu` marker and the repository root on sys.path.

Tests marked `gpu` need a B200 and the built CUDA library; everything else
runs on CPU (`python -m pytest tests -m "not gpu"`).
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built library")
