"""The recurrence's odd shapes under the bounds-checked debug build (GPU only).

``build.py --debug-bounds`` builds ``libtrifusion_b200_bounds.so``, whose recurrence
kernel checks every global access against the tensors' extents (an out-of-range one
records device error 2 and is skipped; nothing traps). ``tests/bounds_cases.py`` runs
T = 1 / 63 / 65, Hq > 1, 2-byte-aligned views, lengths, reversed rows and TMA-staged
long rows through it in a fresh process and requires the error word to stay 0.
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
BOUNDS_LIB = ROOT / "trifusion-fp-kernel_b200" / "trifusion_b200" / "_native" / "libtrifusion_b200_bounds.so"

if not torch.cuda.is_available():
    pytest.skip("needs a CUDA GPU", allow_module_level=True)


def test_odd_shapes_in_the_bounds_checked_build():
    assert BOUNDS_LIB.exists(), "build with `python trifusion-fp-kernel_b200/build.py --debug-bounds`"
    env = dict(os.environ, TRIFUSION_B200_BOUNDS="1")
    r = subprocess.run([sys.executable, str(ROOT / "tests" / "bounds_cases.py")], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0 and "bounds cases ok" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
