"""Shared pytest setup.

* Registers the ``gpu`` marker (tests that need a B200 and the built
  ``libsbfa.so``).
* Puts the package directory on ``sys.path`` so tests import the
  drop-in modules by the same names the upstream project uses
  (``sparse_triton_kernel``, ``fx_compiler_pass``), and the repo root so
  ``oracle`` imports as a package.
"""

from __future__ import annotations

import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "graph-kernel-injection_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libsbfa.so")


@pytest.fixture(scope="session")
def golden_dir() -> str:
    return GOLDEN
