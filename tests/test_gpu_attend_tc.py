"""The tcgen05 gather + attention kernel (``attend_tc_kernel``, selected with LNG_ATTEND_IMPL=tc).

The selection is read once per process, so the memory-layer and drafter parity tests (which cover
its shapes: 136-dim bf16 tokens, 184 / 182 routes, 16 and 4 heads, sequence and window mode) are
re-run in a child process with the variable set.  They compare against the same oracle / golden
fixtures as with the default kernel.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]


def test_memory_and_drafter_parity_with_the_tcgen05_kernel():
    env = dict(os.environ, LNG_ATTEND_IMPL="tc")
    res = subprocess.run([sys.executable, "-m", "pytest", "-q", "-x", "-m", "gpu", "-p", "no:cacheprovider",
                          "tests/test_gpu_memory.py", "tests/test_gpu_drafter.py", "tests/test_gpu_seams.py"],
                         cwd=REPO, env=env, capture_output=True, text=True, timeout=900)
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-2000:]
    assert " passed" in res.stdout
