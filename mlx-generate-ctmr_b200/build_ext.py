"""Build the sm_100a shared library ``ctmr_b200/lib/libctmr_b200.so`` in-tree.

The library is plain CUDA C++ behind the C ABI of ``include/ctmr_b200.h``; it
needs only nvcc (it cross-compiles without a GPU). Objects are compiled in
parallel with relocatable device code and device-linked into one shared object.
Run ``python mlx-generate-ctmr_b200/build_ext.py`` or call :func:`build`.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_ROOT.parent
CSRC = PACKAGE_ROOT / "csrc"
INCLUDE = REPO_ROOT / "include"
BUILD_DIR = PACKAGE_ROOT / "_build"
LIB_PATH = PACKAGE_ROOT / "ctmr_b200" / "lib" / "libctmr_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-rdc=true",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def _nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build ctmr_b200")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(dep.stat().st_mtime > mtime for dep in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``libctmr_b200.so``; returns its path."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_PATH.parent.mkdir(parents=True, exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
    sources = _sources()
    objects = [BUILD_DIR / (src.stem + ".o") for src in sources]

    def compile_one(src: Path, obj: Path) -> None:
        if not force and not _stale(obj, [src, *headers]):
            return
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        list(pool.map(lambda pair: compile_one(*pair), zip(sources, objects, strict=True)))
    if force or _stale(LIB_PATH, objects):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-rdc=true", "-Xcompiler", "-fPIC", *map(str, objects), "-o", str(tmp)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
