"""Builds the sm_100a CUDA library ``libgdn_b200.so`` in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled to an object for ``sm_100a`` only
(``-gencode arch=compute_100a,code=sm_100a``) and linked into one shared
library next to this file.  Objects are rebuilt only when a source or header
is newer than the library.  nvcc cross-compiles, so this runs without a GPU.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
LIB_NAME = "libgdn_b200.so"
LIB_PATH = PKG_DIR / LIB_NAME
OBJ_DIR = PKG_DIR / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3", "-I", str(INCLUDE),
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libgdn_b200.so")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def _compile(nvcc: str, src: Path, extra: list[str]) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compiles the library if needed and returns its path."""
    if not force and not needs_build():
        return LIB_PATH
    nvcc = nvcc_path()
    OBJ_DIR.mkdir(exist_ok=True)
    extra = list(extra_flags or [])
    if verbose:
        extra += ["-Xptxas", "-v"]
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(nvcc, s, extra), srcs))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys
    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
