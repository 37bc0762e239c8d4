"""Shared pytest setup.

* registers the ``gpu`` marker (tests that need a B200 and the built
  ``libqlinear.so``); ``-m "not gpu"`` runs everything else on CPU;
* puts the repository root (for ``oracle``) and the package directory
  ``llm-inference-optimizer_b200/`` (for ``qlinear``) on ``sys.path``.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
PKG_DIR = ROOT / "llm-inference-optimizer_b200"
for p in (str(ROOT), str(PKG_DIR)):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200) and the built libqlinear.so")


def pytest_sessionstart(session):
    """Build libqlinear.so in-tree if it is missing (nvcc cross-compiles for
    sm_100a without a GPU).  A stale-but-present library is left alone."""
    from qlinear import _build
    if not _build.OUT.exists():
        _build.build()
