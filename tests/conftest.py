"""Shared test setup.

* Registers the ``gpu`` marker: tests that need a CUDA device (run on a B200
  with ``pytest -m gpu``); everything else runs on CPU (``-m "not gpu"``).
* Puts the drop-in package (``kitty-kv_b200/``) and the repository root (for
  the ``oracle`` checker) on ``sys.path``.
* Loads the golden vectors recorded from the reference implementation.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent
PKG = REPO / "kitty-kv_b200"
GOLDEN = Path(__file__).resolve().parent / "golden"
for p in (str(PKG), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


@pytest.fixture(scope="session")
def golden_npz():
    with np.load(GOLDEN / "golden_small.npz") as z:
        return {k: z[k] for k in z.files}


@pytest.fixture(scope="session")
def golden_manifest():
    return json.loads((GOLDEN / "golden_manifest.json").read_text())


def small_case_names(store, kind):
    return sorted({k.split("/")[1] for k in store if k.startswith(kind + "/")})


def sha(a) -> str:
    import hashlib
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def meta_by_value(a) -> np.ndarray:
    """Metadata compared by value: +0.0 and -0.0 are equal (the reference's
    zero-point sign depends on which SIMD lane computed it)."""
    return np.asarray(a).astype(np.float32) + np.float32(0.0)
