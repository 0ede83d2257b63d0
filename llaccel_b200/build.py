"""Builds the CUDA backend in-tree: llaccel_b200/csrc/*.cu -> llaccel_b200/_lib/libllx.so.

    python -m llaccel_b200.build [--force]

Compiled for sm_100a only (B200).  nvcc cross-compiles without a GPU, so this runs on any
host with the CUDA toolkit.  The build is skipped when the library is newer than every
source file.
"""
from __future__ import annotations

import argparse
import fcntl
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "_lib"
LIB = LIBDIR / "libllx.so"
INCLUDE = PKG.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build llaccel_b200")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def deps() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + \
        sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile if any source is newer than the library.  Processes that start together (one
    per GPU rank) serialise on a lock file: the first rebuilds, the others find the library
    up to date once they hold the lock."""
    if not force and up_to_date():
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    with open(LIBDIR / ".build.lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not force and up_to_date():
                return LIB
            return _compile(verbose)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)


def _compile(verbose: bool) -> Path:
    objdir = PKG / "_build" / str(os.getpid())
    objdir.mkdir(parents=True, exist_ok=True)
    objs = []
    for src in sources():
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr)
        objs.append(str(obj))
    tmp = LIB.with_suffix(f".so.{os.getpid()}.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *objs, "-lcuda", "-ldl"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    shutil.rmtree(objdir, ignore_errors=True)
    return LIB


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(a.force, a.verbose))


if __name__ == "__main__":
    main(sys.argv[1:])
