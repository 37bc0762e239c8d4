"""Installs the unmodified reference into baseline/_ref (test and baseline
infrastructure, not product code).

The reference is a plain source tree (``src/`` with the kernels, the
quantization modules and the engines) without packaging metadata, so
``pip install <reference>`` refuses it.  This script copies the tree to a
temporary directory, adds a minimal pyproject.toml that lists the ``src``
packages — the sources themselves are not changed — and installs that copy
with pip, offline, into baseline/_ref.  The result travels with the
repository snapshot to GPU machines, where the bench's CPU legs time the
reference's own ``w4a16_reference`` and the engine drop-in tests run the
reference's engines over this build's modules.

    python oracle/install_reference.py [--force]

The reference's location is BASELINE.json's ``reference_path``.  Nothing is
done when that directory is absent (as on GPU machines) or when baseline/_ref
already holds the install.
"""
from __future__ import annotations

import json
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
TARGET = ROOT / "baseline" / "_ref"
PACKAGES = ["src", "src.engine", "src.kernels", "src.kv_cache", "src.quantization"]
PYPROJECT = """[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "llm-inference-optimizer-reference"
version = "0.0.0"

[tool.setuptools]
packages = {packages}
"""


def reference_path() -> Path | None:
    try:
        return Path(json.loads((ROOT / "BASELINE.json").read_text())["reference_path"])
    except Exception:
        return None


def installed() -> bool:
    return (TARGET / "src" / "kernels" / "w4a16_matmul_triton.py").exists()


def install(force: bool = False, quiet: bool = True) -> str:
    """Returns a one-line outcome."""
    ref = reference_path()
    if ref is None or not (ref / "src").is_dir():
        return "reference source tree not present here; baseline/_ref left as it is"
    if installed() and not force:
        return "baseline/_ref already installed"
    with tempfile.TemporaryDirectory(prefix="refpkg_") as tmp:
        pkg = Path(tmp) / "pkg"
        shutil.copytree(ref / "src", pkg / "src", ignore=shutil.ignore_patterns("__pycache__"))
        (pkg / "pyproject.toml").write_text(PYPROJECT.format(packages=json.dumps(PACKAGES)))
        if TARGET.exists():
            shutil.rmtree(TARGET)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", str(TARGET), str(pkg)]
        res = subprocess.run(cmd, capture_output=quiet, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"pip install of the reference failed ({res.returncode}):\n"
                               f"{res.stdout}\n{res.stderr}")
    return "installed into baseline/_ref"


if __name__ == "__main__":
    print(install(force="--force" in sys.argv, quiet=False))
