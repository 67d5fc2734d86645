"""Build libragged_b200.so in-tree with nvcc for sm_100a (no GPU needed).

    python ragged-mlir_b200/build.py [--force] [-j JOBS]

Every ``csrc/*.cu`` file is compiled to an object under ``_build/`` in
parallel, then linked into ``ragged/_lib/libragged_b200.so`` next to the
Python package that loads it.  Objects are rebuilt when their source or any
``csrc/*.cuh|*.h`` header (or ``include/*.h``) is newer.
"""
from __future__ import annotations

import argparse
from concurrent.futures import ThreadPoolExecutor
import os
from pathlib import Path
import shutil
import subprocess
import sys

PACKAGE_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_ROOT.parent
CSRC = PACKAGE_ROOT / "csrc"
BUILD = PACKAGE_ROOT / "_build"
LIBRARY = PACKAGE_ROOT / "ragged" / "_lib" / "libragged_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills", "-I", str(REPO_ROOT / "include")]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found")
    return path


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((REPO_ROOT / "include").glob("*.h"))


def _stale(target: Path, sources: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(source.stat().st_mtime > mtime for source in sources)


def _compile(source: Path, force: bool, verbose: bool) -> Path:
    obj = BUILD / (source.stem + ".o")
    if force or _stale(obj, [source, *_headers()]):
        cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(source), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stdout}\n{result.stderr}")
        if verbose and result.stderr:
            print(result.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compile and link; returns the library path."""
    BUILD.mkdir(parents=True, exist_ok=True)
    LIBRARY.parent.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    jobs = jobs or min(len(sources), os.cpu_count() or 4)
    with ThreadPoolExecutor(jobs) as pool:
        objects = list(pool.map(lambda s: _compile(s, force, verbose), sources))
    if force or _stale(LIBRARY, objects):
        tmp = LIBRARY.with_suffix(f".{os.getpid()}.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objects), "-lcudart"]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode:
            raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("-j", "--jobs", type=int)
    parser.add_argument("-v", "--verbose", action="store_true", help="print ptxas resource usage")
    args = parser.parse_args()
    print(build(args.force, args.jobs, args.verbose))


if __name__ == "__main__":
    main()
