"""pytest configuration: markers, repo paths, and the shared fixtures of the suite.

``-m gpu`` tests need a B200 and the built CUDA library; everything else runs on the CPU.
Tests marked ``reference`` import the reference checkout (read-only) when it is present
(``LNGRAM_REFERENCE``, else a checkout named ``reference`` beside this repository) and are
skipped when it is not.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
# the reference checkout: LNGRAM_REFERENCE, else a directory named "reference" beside this repository
REFERENCE = Path(os.environ.get("LNGRAM_REFERENCE") or (REPO.parent / "reference"))
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built lngram_b200 library")
    config.addinivalue_line("markers", "reference: imports the reference checkout; skipped without it")
    config.addinivalue_line("markers", "slow: longer CPU test")


def pytest_collection_modifyitems(config, items):
    have_ref = (REFERENCE / "ffnmem" / "memory" / "lngram_v2.py").exists()
    for item in items:
        if "reference" in item.keywords and not have_ref:
            item.add_marker(pytest.mark.skip(reason="reference checkout not present"))


@pytest.fixture(scope="session")
def golden():
    """Loader of the committed golden fixtures: golden('memory_tiny') -> dict of arrays."""
    cache = {}

    def load(name: str) -> dict:
        if name not in cache:
            with np.load(GOLDEN / f"{name}.npz") as z:
                cache[name] = {k: z[k] for k in z.files}
        return cache[name]

    return load


@pytest.fixture(scope="session")
def lngram():
    """The ``lngram-decode_b200`` package (imported through ``__graft_entry__``)."""
    from __graft_entry__ import load_package

    return load_package()


@pytest.fixture(scope="session")
def reference_path():
    # appended, so this repository's own top-level names (``tests``, ``oracle``) keep precedence
    # over the reference's packages of the same name
    if str(REFERENCE) not in sys.path:
        sys.path.append(str(REFERENCE))
    return REFERENCE
