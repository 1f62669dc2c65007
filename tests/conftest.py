"""Test configuration: the `gpu` marker and import paths.

`-m "not gpu"` runs the oracle pins, host logic and C-ABI load checks on a
CPU-only machine; `-m gpu` runs the CUDA parity tests on a B200.
"""

import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "trifusion-fp-kernel_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100) GPU")
