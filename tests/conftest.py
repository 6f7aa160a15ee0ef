"""Shared pytest setup: the `gpu` marker and import paths.

Tests marked ``gpu`` need a CUDA device (a B200); everything else runs on the
CPU (oracle checks, golden fixtures, host logic, ABI symbol checks).
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")
