"""Build libremora_b200.so in-tree with nvcc for sm_100a.

Usage: python -m remora_b200.csrc.build  (or build() from Python).  Object
files go to remora_b200/csrc/_build/; the shared library lands next to the
package so a plain snapshot of the repository carries it.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
PKG = HERE.parent
ROOT = PKG.parent
OUT = PKG / "libremora_b200.so"
BUILD = HERE / "_build"

SOURCES = sorted(HERE.glob("*.cu"))

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    f"-I{ROOT / 'include'}",
    "--expt-relaxed-constexpr",
]


def _host_compiler() -> list[str]:
    # nvcc needs a host g++; prefer the system one over a CC/CXX from the
    # environment that may lack pieces of its runtime.
    for cand in ("/usr/bin/g++", shutil.which("g++")):
        if cand and Path(cand).exists():
            return ["-ccbin", cand]
    return []


def _needs_rebuild(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *HERE.glob("*.cuh"), *(ROOT / "include").glob("*.h")]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps if d.exists())


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if _needs_rebuild(obj, src):
        cmd = [NVCC, *_host_compiler(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return obj


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    if not OUT.exists() or any(o.stat().st_mtime > OUT.stat().st_mtime for o in objs):
        cmd = [
            NVCC,
            *_host_compiler(),
            *ARCH,
            "-shared",
            "-o",
            str(OUT),
            *map(str, objs),
            f"-L{CUDA_HOME / 'lib64'}",
            "-lnvrtc",
            f"-Xlinker=-rpath,{CUDA_HOME / 'lib64'}",
        ]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
