"""Build the sm_100a shared library ``libmingru_scan.so`` in-tree.

Every ``csrc/*.cu`` file is compiled by ``nvcc`` for ``sm_100a`` only (no PTX
for other architectures: this library targets B200) and linked into one
shared object next to this file, so the built library travels with the
source tree instead of living in a per-user JIT cache. Usage::

    python -m mingru_b200.build          # incremental
    python -m mingru_b200.build --force  # rebuild everything
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
INCLUDE = PKG_DIR.parent / "include"
OBJ_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "libmingru_scan.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++20",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3",
    "-I",
    str(INCLUDE),
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")
    return cand


def _deps(src: Path) -> list[Path]:
    return [src, *CSRC.glob("*.cuh"), *INCLUDE.glob("*.h")]


def _compile(src: Path, force: bool, verbose: bool) -> Path:
    obj = OBJ_DIR / (src.stem + ".o")
    if not force and obj.exists():
        newest = max(p.stat().st_mtime for p in _deps(src))
        if obj.stat().st_mtime >= newest:
            return obj
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every kernel file and link ``libmingru_scan.so``; return its path."""
    OBJ_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError(f"no CUDA sources under {CSRC}")
    workers = max(1, min(len(sources), os.cpu_count() or 1))
    with cf.ThreadPoolExecutor(workers) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), sources))
    if (
        force
        or not LIB_PATH.exists()
        or LIB_PATH.stat().st_mtime < max(o.stat().st_mtime for o in objs)
    ):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc_path(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas register usage")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
