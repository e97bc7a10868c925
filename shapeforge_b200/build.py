"""Build ``libsfcuda.so`` (the sm_100a kernels + C ABI) in-tree with nvcc.

Usage: ``python -m shapeforge_b200.build [--force] [-j N]``.  Objects go to
``shapeforge_b200/_build/``; the shared library lands next to this file so it travels with the
source tree.  Only objects whose sources (or shared headers) changed are rebuilt.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libsfcuda.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-warn-spills",
]


def nvcc() -> str:
    """Path of nvcc (``$CUDA_HOME/bin/nvcc`` or on PATH)."""
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(home) / "bin" / "nvcc"
    if cand.is_file():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def _compile(src: Path, obj: Path, extra: list[str]) -> tuple[Path, str]:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
    return obj, proc.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False, extra: list[str] | None = None) -> Path:
    """Compile every ``csrc/*.cu`` for sm_100a and link ``libsfcuda.so``; return its path."""
    BUILD.mkdir(exist_ok=True)
    deps = _headers()
    work = []
    for src in _sources():
        obj = BUILD / (src.stem + ".o")
        if force or _stale(obj, src, deps):
            work.append((src, obj))
    jobs = jobs or min(8, os.cpu_count() or 1)
    if work:
        with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as pool:
            futs = [pool.submit(_compile, s, o, list(extra or [])) for s, o in work]
            for fut in futs:
                obj, log = fut.result()
                if verbose and log.strip():
                    print(f"[{obj.name}]\n{log}", file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in _sources()]
    if force or work or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{proc.stdout}\n{proc.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas output (-Xptxas -v is added)")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.verbose else []
    path = build(force=args.force or args.verbose, jobs=args.jobs, verbose=args.verbose, extra=extra)
    print(path)


if __name__ == "__main__":
    main()
