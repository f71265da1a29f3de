"""Build librabbit_cuda.so (sm_100a) in-tree with nvcc.

    python -m rabbit_b200.build [--force]

Each csrc/*.cu is compiled to an object under rabbit_b200/_build/ and linked
into rabbit_b200/librabbit_cuda.so with the CUDA runtime linked statically,
so the library only needs the NVIDIA driver at run time. Objects are rebuilt
when their source or any header changed.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "librabbit_cuda.so"
BUILD = PKG / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _flags() -> list[str]:
    return ARCH + ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                   "-I" + str(ROOT / "include"), "--expt-relaxed-constexpr", "-Xptxas",
                   "-warn-spills"]


def _stale(obj: Path, src: Path, headers: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *headers])


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(
        (ROOT / "include").glob("*.h"))
    objs = []
    changed = force or not OUT.exists()
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _stale(obj, src, headers):
            cmd = [nvcc(), *_flags(), "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.check_call(cmd)
            changed = True
    if changed or any(o.stat().st_mtime > OUT.stat().st_mtime for o in objs):
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp),
               *map(str, objs), "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        os.replace(tmp, OUT)
    return OUT


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(a.force, a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
