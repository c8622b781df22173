"""Builds ``libpicotron_b200.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

Usage: ``python -m picotron_b200.build [--force] [--ptxas-verbose]``.

Every ``csrc/*.cu`` file is compiled to an object under ``picotron_b200/_build/`` and the
objects are linked into ``picotron_b200/libpicotron_b200.so``. The CUDA runtime is linked
statically, so the library depends only on the driver; kernels launch on the caller's
stream handle, which is a driver-level object shared with PyTorch's runtime.
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
REPO_DIR = PACKAGE_DIR.parent
CSRC_DIR = PACKAGE_DIR / "csrc"
INCLUDE_DIR = REPO_DIR / "include"
BUILD_DIR = PACKAGE_DIR / "_build"
LIBRARY_NAME = "libpicotron_b200.so"
LIBRARY_PATH = PACKAGE_DIR / LIBRARY_NAME

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-DNDEBUG",
]


def find_nvcc() -> str:
    """Locate nvcc: $CUDA_HOME/bin, then PATH, then /usr/local/cuda/bin."""

    candidates = []
    if os.environ.get("CUDA_HOME"):
        candidates.append(Path(os.environ["CUDA_HOME"]) / "bin" / "nvcc")
    which = shutil.which("nvcc")
    if which:
        candidates.append(Path(which))
    candidates.append(Path("/usr/local/cuda/bin/nvcc"))
    for candidate in candidates:
        if candidate.is_file():
            return str(candidate)
    raise RuntimeError("nvcc not found; set CUDA_HOME or put nvcc on PATH")


def _sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def _newest_mtime(paths: list[Path]) -> float:
    return max((p.stat().st_mtime for p in paths), default=0.0)


def _compile(nvcc: str, src: Path, obj: Path, ptxas_verbose: bool) -> tuple[Path, str]:
    cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, f"-I{INCLUDE_DIR}", "-c", str(src), "-o", str(obj)]
    if ptxas_verbose:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stdout + proc.stderr


def build(force: bool = False, ptxas_verbose: bool = False, verbose: bool = False) -> Path:
    """Compile the sources that changed and relink; returns the library path."""

    nvcc = find_nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    header_mtime = _newest_mtime(_headers())
    jobs = []
    objects = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        stale = (
            force
            or ptxas_verbose
            or not obj.exists()
            or obj.stat().st_mtime < max(src.stat().st_mtime, header_mtime)
        )
        if stale:
            jobs.append((src, obj))
    logs = []
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 1)
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
            futures = [pool.submit(_compile, nvcc, s, o, ptxas_verbose) for s, o in jobs]
            for fut in futures:
                obj, log = fut.result()
                logs.append((obj.name, log))
    relink = (
        force
        or bool(jobs)
        or not LIBRARY_PATH.exists()
        or LIBRARY_PATH.stat().st_mtime < _newest_mtime(objects)
    )
    if relink:
        tmp = LIBRARY_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp)]
        cmd += [str(o) for o in objects]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIBRARY_PATH)
    if verbose or ptxas_verbose:
        for name, log in logs:
            if log.strip():
                print(f"--- {name}\n{log}", file=sys.stderr)
    return LIBRARY_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true", help="rebuild everything")
    parser.add_argument("--ptxas-verbose", action="store_true", help="print -Xptxas -v output")
    args = parser.parse_args()
    path = build(force=args.force, ptxas_verbose=args.ptxas_verbose, verbose=True)
    print(path)


if __name__ == "__main__":
    main()
