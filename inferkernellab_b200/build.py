"""Build the sm_100a shared library ``_lib/libb200_paged_attn.so`` in-tree.

``python -m inferkernellab_b200.build`` (or ``build()``) compiles every
``csrc/*.cu`` with nvcc for ``sm_100a`` only, in parallel, and links them into
one shared library with the C ABI of ``include/b200_paged_attn.h``.  The
library is rebuilt when a source or header is newer than it.  nvcc
cross-compiles, so this works on a machine without a GPU.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
OUT_DIR = PKG / "_lib"
LIB_NAME = "libb200_paged_attn.so"
LIB_PATH = OUT_DIR / LIB_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
    "-Xptxas", "-O3",
]


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = Path("/usr/local/cuda/bin/nvcc")
    if default.exists():
        return str(default)
    raise RuntimeError("nvcc not found: the sm_100a kernels cannot be built")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _inputs() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(
        INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in _inputs())


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile and link the library if it is missing or stale; return its path."""
    if not force and not needs_build():
        return LIB_PATH
    nvcc = _nvcc()
    obj_dir = OUT_DIR / "obj"
    obj_dir.mkdir(parents=True, exist_ok=True)
    jobs = jobs or min(8, os.cpu_count() or 4)

    def compile_one(src: Path) -> Path:
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd += ["-Xptxas", "-v"]
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        if verbose and res.stderr:
            print(res.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=jobs) as pool:
        objs = list(pool.map(compile_one, _sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> None:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="show nvcc commands and -Xptxas -v")
    args = parser.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    main(sys.argv[1:])
