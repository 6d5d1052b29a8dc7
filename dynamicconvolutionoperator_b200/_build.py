"""Build ``libddpm_b200.so`` in-tree with nvcc for sm_100a.

Every ``csrc/*.cu`` file is compiled separately (in parallel, skipped when the
object is newer than the source and the shared headers) into ``_build/`` and
linked into ``dynamicconvolutionoperator_b200/libddpm_b200.so``. The library is
a plain C-ABI shared object (see ``include/ddpm_b200.h``); Python loads it with
ctypes, so no torch headers or torch ABI are involved.

Usage: ``python -m dynamicconvolutionoperator_b200._build [--force] [--debug]``.
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
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build"
LIB_PATH = PKG_DIR / "libddpm_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
BASE_FLAGS = [
    "-std=c++17",
    "-O3",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3,-fvisibility=hidden",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; set NVCC or add CUDA's bin directory to PATH")
    return cand


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(obj: Path, src: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *deps])


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library; returns its path."""
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if not sources:
        raise RuntimeError(f"no CUDA sources under {CSRC}")
    deps = _headers()
    extra = ["-DDDPM_CHECK_BOUNDS", "-G0"] if debug else []
    flags = ARCH_FLAGS + BASE_FLAGS + extra + [f"-I{INCLUDE}", f"-I{CSRC}"]

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.stem + ".o")
        if force or _stale(obj, src, deps):
            cmd = [nvcc, *flags, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            res = subprocess.run(cmd, capture_output=True, text=True)
            if res.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
        return obj

    workers = min(len(sources), os.cpu_count() or 4)
    with cf.ThreadPoolExecutor(max_workers=workers) as pool:
        objs = list(pool.map(compile_one, sources))

    if force or not LIB_PATH.exists() or any(
        o.stat().st_mtime > LIB_PATH.stat().st_mtime for o in objs
    ):
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true", help="device-side bounds checks")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args(argv)
    path = build(force=args.force, debug=args.debug, verbose=args.verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
