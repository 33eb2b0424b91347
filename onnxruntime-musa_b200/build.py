"""Build recipe of libmoe_b200.so (sm_100a) -- run by ``__graft_entry__.build()``.

Each ``csrc/*.cu`` is compiled by nvcc for ``compute_100a``/``sm_100a`` into
``_build/`` and linked into ``lib/libmoe_b200.so``; only the ``moe_b200_*`` C ABI is
exported (``csrc/libmoe_b200.lds``).  CUDA runtime is linked statically, so the
library needs only the driver at run time.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

HERE = pathlib.Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "lib" / "libmoe_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
              "--expt-relaxed-constexpr", "-Xptxas", "-O3"]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found")
    return cand


def _compile(src: pathlib.Path, verbose_ptxas: bool) -> pathlib.Path:
    obj = BUILD / (src.stem + ".o")
    deps = [src] + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + \
        sorted((HERE.parent / "include").glob("*.h"))
    if obj.exists() and obj.stat().st_mtime >= max(d.stat().st_mtime for d in deps):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd[1:1] = ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
    if verbose_ptxas:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose_ptxas: bool = False) -> pathlib.Path:
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), sources))
    newest = max(o.stat().st_mtime for o in objs)
    lds = CSRC / "libmoe_b200.lds"
    if LIB.exists() and LIB.stat().st_mtime >= max(newest, lds.stat().st_mtime):
        return LIB
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs),
           "-Xlinker", f"--version-script={lds}", "-lrt"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose_ptxas="-v" in sys.argv))
