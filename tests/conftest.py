"""Shared test configuration.

Tests marked ``gpu`` need a CUDA device (a B200 for this build) and call the
CUDA library through its C ABI; everything else runs on CPU.
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device and the built CUDA library")
