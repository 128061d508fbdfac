"""Installs the reference benchmark package (transformer_benchmark) into baseline/_ref.

The reference checkout is a flat project with several top-level folders (orchestrator/,
research/, tests/, transformer_benchmark/) and no build-system table, so
`pip install <checkout>` stops at setuptools' package discovery. This recipe installs the one
package the benchmark CLI imports, unmodified: it copies `transformer_benchmark/` into a
temporary project whose only addition is a pyproject.toml naming that package (and its .cu
sources as package data), then runs the offline pip install into baseline/_ref.

baseline/_ref is ignored by git (it is the reference's code, not this project's) but travels with
the source tree to the GPU box, where tests/test_gpu_reference_runner.py drives the reference's
own runner with this package's UserOptimizedTransformer in the candidate slot.

Usage: python baseline/install_reference.py [--reference /path/to/checkout]
       (default: $REFERENCE_ROOT)
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"

PYPROJECT = """\
[build-system]
requires = ["setuptools"]
build-backend = "setuptools.build_meta"

[project]
name = "tiktok-techjam-2026-track-3-benchmark"
version = "0.1.0"
requires-python = ">=3.12"

[tool.setuptools]
packages = ["transformer_benchmark"]

[tool.setuptools.package-data]
transformer_benchmark = ["*.cu"]
"""


def install(reference: Path) -> Path:
    src = reference / "transformer_benchmark"
    if not (src / "runner.py").is_file():
        raise SystemExit(f"{reference} is not a reference checkout (no transformer_benchmark/runner.py)")
    with tempfile.TemporaryDirectory(prefix="refpkg_") as tmp:
        proj = Path(tmp)
        shutil.copytree(src, proj / "transformer_benchmark", ignore=shutil.ignore_patterns("__pycache__"))
        (proj / "pyproject.toml").write_text(PYPROJECT)
        if TARGET.exists():
            shutil.rmtree(TARGET)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--no-deps",
               "--find-links", "/opt/wheelhouse", "--target", str(TARGET), str(proj)]
        subprocess.run(cmd, check=True)
    return TARGET


def main() -> None:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--reference", default=os.environ.get("REFERENCE_ROOT"),
                   help="reference checkout (default: $REFERENCE_ROOT)")
    args = p.parse_args()
    if not args.reference:
        raise SystemExit("pass --reference or set REFERENCE_ROOT")
    print(install(Path(args.reference)))


if __name__ == "__main__":
    main()
