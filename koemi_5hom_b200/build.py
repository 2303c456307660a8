"""Build recipe for ``libkoemi_b200.so``, the sm_100a kernel library.

Every ``csrc/*.cu`` translation unit is compiled by nvcc for
``-gencode arch=compute_100a,code=sm_100a`` into an object under ``_build/``
(skipped when the object is newer than its sources), and the objects are
linked into ``lib/libkoemi_b200.so`` with a static CUDA runtime, so the
library depends on nothing but the driver. nvcc cross-compiles without a GPU.

Run ``python -m koemi_5hom_b200.build`` (or call :func:`build`).
"""
from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
SOURCE_DIR = PACKAGE_DIR / "csrc"
INCLUDE_DIR = PACKAGE_DIR.parent / "include"
BUILD_DIR = PACKAGE_DIR.parent / "_build"
LIBRARY_PATH = PACKAGE_DIR / "lib" / "libkoemi_b200.so"

ARCH_FLAGS = ("-gencode", "arch=compute_100a,code=sm_100a")
NVCC_FLAGS = (
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-Xptxas",
    "-warn-spills",
)


def find_nvcc() -> str:
    candidates = [os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"]
    for candidate in candidates:
        if candidate and Path(candidate).is_file():
            return candidate
    raise RuntimeError("nvcc was not found; set NVCC or put the CUDA toolkit on PATH")


def _headers() -> list[Path]:
    return sorted(SOURCE_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def _compile(nvcc: str, source: Path, verbose: bool) -> Path:
    target = BUILD_DIR / (source.stem + ".o")
    newest_input = max(p.stat().st_mtime for p in [source, *_headers(), Path(__file__)])
    if target.exists() and target.stat().st_mtime >= newest_input:
        return target
    command = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE_DIR), "-c", str(source), "-o", str(target)]
    if verbose:
        print(" ".join(command), flush=True)
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed on {source.name}:\n{result.stdout}\n{result.stderr}")
    if verbose and (result.stdout or result.stderr):
        print(result.stdout + result.stderr, flush=True)
    return target


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile every kernel translation unit and link the shared library."""
    nvcc = find_nvcc()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIBRARY_PATH.parent.mkdir(parents=True, exist_ok=True)
    sources = sorted(SOURCE_DIR.glob("*.cu"))
    if not sources:
        raise RuntimeError(f"no CUDA sources under {SOURCE_DIR}")
    workers = jobs or min(len(sources), os.cpu_count() or 4)
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
        objects = list(pool.map(lambda s: _compile(nvcc, s, verbose), sources))
    newest_object = max(o.stat().st_mtime for o in objects)
    if LIBRARY_PATH.exists() and LIBRARY_PATH.stat().st_mtime >= newest_object:
        return LIBRARY_PATH
    temporary = LIBRARY_PATH.with_suffix(".so.tmp")
    command = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(temporary),
               *map(str, objects)]
    if verbose:
        print(" ".join(command), flush=True)
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"linking libkoemi_b200.so failed:\n{result.stdout}\n{result.stderr}")
    os.replace(temporary, LIBRARY_PATH)
    return LIBRARY_PATH


def main(argv: list[str] | None = None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("-v", "--verbose", action="store_true")
    parser.add_argument("-j", "--jobs", type=int, default=None)
    arguments = parser.parse_args(argv)
    path = build(verbose=arguments.verbose, jobs=arguments.jobs)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
