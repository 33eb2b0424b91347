#!/usr/bin/env python3
"""Builds a platform wheel of the package.

The wheel installs the importable module ``onnxruntime_musa_b200`` (this directory's
``__init__.py`` and ``ep.py``) with the built library ``lib/libmoe_b200.so`` and the C
header ``include/moe_b200.h`` beside it, so ``get_library_path()`` works from the install
as it does in-tree.  It plays the role of the reference's wheel builder
(``musa/ep/python/build_wheel.py``: a staging directory with the package and the plugin
binary, a generated ``pyproject.toml``, ``pip wheel --no-deps --no-build-isolation``, a
``py3-none-<platform>`` tag); the package layout and metadata here are this project's own.

    python onnxruntime-musa_b200/build_wheel.py --output_dir dist [--version 0.1.0]

Build the library first (``build.py``).  The CUDA runtime and driver libraries that the
library links against are system dependencies; they are not put into the wheel.
"""

from __future__ import annotations

import argparse
import re
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent
MODULE = "onnxruntime_musa_b200"
DEFAULT_NAME = "onnxruntime-b200-moe"
DEFAULT_VERSION = "0.1.0"

SETUP_PY = '''\
"""Platform wheel: the package carries a prebuilt shared library."""
from setuptools import setup
from setuptools.command.bdist_wheel import bdist_wheel
from setuptools.dist import Distribution


class PlatformWheel(bdist_wheel):
    def get_tag(self):
        _, _, plat = super().get_tag()
        return "py3", "none", plat


class BinaryDistribution(Distribution):
    def has_ext_modules(self):
        return True


setup(distclass=BinaryDistribution, cmdclass={"bdist_wheel": PlatformWheel})
'''

PYPROJECT = '''\
[build-system]
requires = ["setuptools>=64", "wheel"]
build-backend = "setuptools.build_meta"

[project]
name = "{name}"
version = "{version}"
description = "B200 (sm_100a) MoE / QMoE hot path behind an ONNX Runtime plugin EP boundary"
requires-python = ">=3.10"
dependencies = []

[project.optional-dependencies]
torch = ["torch"]

[tool.setuptools]
packages = ["{module}"]
include-package-data = false

[tool.setuptools.package-data]
{module} = ["lib/*.so", "include/*.h", "py.typed"]
'''


def stage(staging: Path, name: str, version: str) -> None:
    lib = PKG_DIR / "lib" / "libmoe_b200.so"
    if not lib.is_file():
        raise FileNotFoundError(f"{lib} is missing: build the library first (build.py)")
    pkg = staging / MODULE
    (pkg / "lib").mkdir(parents=True)
    (pkg / "include").mkdir()
    for src in ("__init__.py", "ep.py"):
        shutil.copy2(PKG_DIR / src, pkg / src)
    shutil.copy2(lib, pkg / "lib" / lib.name)
    shutil.copy2(ROOT / "include" / "moe_b200.h", pkg / "include" / "moe_b200.h")
    (pkg / "py.typed").write_text("")
    (staging / "setup.py").write_text(SETUP_PY)
    (staging / "pyproject.toml").write_text(
        PYPROJECT.format(name=name, version=version, module=MODULE))


def build(output_dir: Path, name: str = DEFAULT_NAME, version: str = DEFAULT_VERSION) -> Path:
    """Builds the wheel into output_dir and returns its path."""
    if not re.fullmatch(r"[A-Za-z0-9][A-Za-z0-9._-]*", name):
        raise ValueError(f"invalid distribution name {name!r}")
    if not re.fullmatch(r"\d+(\.\d+)*([ab]|rc)?\d*(\.dev\d+)?", version):
        raise ValueError(f"invalid version {version!r}")
    output_dir.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory(prefix="moe_b200_wheel_") as tmp:
        staging = Path(tmp) / "src"
        stage(staging, name, version)
        out = Path(tmp) / "out"
        subprocess.run([sys.executable, "-m", "pip", "wheel", str(staging), "--wheel-dir",
                        str(out), "--no-deps", "--no-build-isolation", "--no-index", "-q"],
                       check=True)
        wheels = list(out.glob("*.whl"))
        if len(wheels) != 1:
            raise RuntimeError(f"expected one wheel, got {wheels}")
        dest = output_dir / wheels[0].name
        shutil.copy2(wheels[0], dest)
    return dest


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--output_dir", type=Path, required=True)
    ap.add_argument("--package_name", default=DEFAULT_NAME)
    ap.add_argument("--version", default=DEFAULT_VERSION)
    args = ap.parse_args()
    print(build(args.output_dir, args.package_name, args.version))


if __name__ == "__main__":
    main()
