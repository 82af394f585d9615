"""Build libexpertrelay_b200.so in-tree with nvcc for sm_100a.

    python -m expertrelay_b200.build [--force] [--verbose]

Each csrc/*.cu compiles to an object under _build/ (in parallel, skipped
when up to date with its sources and headers), then they link into
expertrelay_b200/libexpertrelay_b200.so with the CUDA runtime linked
statically, so the library depends on no particular libcudart at run time.
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
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libexpertrelay_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put /usr/local/cuda/bin on PATH)")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd), flush=True)
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        sys.stderr.write(proc.stdout + proc.stderr)
        raise RuntimeError(f"command failed ({proc.returncode}): {' '.join(cmd[:4])} ...")
    if verbose and (proc.stdout or proc.stderr):
        sys.stderr.write(proc.stdout + proc.stderr)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link the shared library.
    Returns the library path."""
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    cc = nvcc()
    jobs = []
    objects = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objects.append(obj)
        if force or _stale(obj, [src, *headers]):
            cmd = [cc, *FLAGS, *ARCH, f"-I{INCLUDE}", "-c", str(src), "-o", str(obj)]
            if ptxas_info:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    if jobs:
        with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(lambda c: _run(c, verbose), jobs))
    if force or jobs or _stale(LIB, objects):
        tmp = LIB.with_suffix(".so.tmp")
        _run([cc, "-shared", *ARCH, "-o", str(tmp), *map(str, objects)], verbose)
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print register / shared-memory use per kernel")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))


if __name__ == "__main__":
    main()
