"""Shared fixtures and markers.

``-m gpu`` tests need a B200 and the built ``libmdlc_b200.so``; everything else
runs on CPU. Golden fixtures live in ``tests/golden`` (made by
``tests/golden/make_golden.py`` from the reference implementation).
"""

from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 and the built sm_100a library")


@pytest.fixture
def rng():
    return np.random.default_rng(1234)


def golden(case: str) -> dict:
    with np.load(os.path.join(GOLDEN, f"{case}.npz")) as z:
        return {k: z[k] for k in z.files}
