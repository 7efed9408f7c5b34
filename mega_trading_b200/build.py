"""Build the sm_100a shared library ``libmtb200.so`` in-tree.

Every ``csrc/*.cu`` file is compiled separately with nvcc for
``compute_100a``/``sm_100a`` (objects under ``_build/``, rebuilt when the file or
a header is newer) and linked into ``mega_trading_b200/lib/libmtb200.so`` with
the CUDA runtime linked statically, so the library loads on hosts without a
GPU driver (the C ABI can then be inspected; kernels need a B200).

Usage: ``python -m mega_trading_b200.build [--force] [--verbose]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures as futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libmtb200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-DNDEBUG",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the B200 library needs the CUDA 12.9 toolkit")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, obj: Path, verbose: bool) -> tuple[Path, str]:
    cmd = [nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-Xptxas", "-v", "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    log = proc.stdout + proc.stderr
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{log}")
    (obj.with_suffix(".ptxas.txt")).write_text(log)
    if verbose:
        print(log)
    return src, log


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every csrc/*.cu for sm_100a and link libmtb200.so; return its path."""
    BUILD.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    jobs = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, *headers]):
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), max(1, os.cpu_count() or 1))
        with futures.ThreadPoolExecutor(max_workers=workers) as pool:
            for fut in [pool.submit(_compile, s, o, verbose) for s, o in jobs]:
                fut.result()
    if force or jobs or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}{proc.stderr}")
    return LIB


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
