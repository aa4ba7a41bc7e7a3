"""Build libwhallm_moe.so in-tree: every .cu of csrc/ compiled for sm_100a.

Run ``python -m whallm_b200.build`` (or ``__graft_entry__.build()``).  Objects
go to ``_build/`` at the repository root; the shared library lands next to
this file so that it travels with the source tree.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libwhallm_moe.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-I", str(ROOT / "include"), "-I", str(CSRC),
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cuda = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if cuda.exists():
        return str(cuda)
    raise RuntimeError("nvcc not found: set CUDA_HOME or put nvcc on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src, *CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *(ROOT / "include").glob("*.h")]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def compile_one(src: Path, verbose: bool = False, extra: list[str] | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    obj = BUILD / (src.stem + ".o")
    if not _stale(obj, src) and not extra:
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *(extra or []), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout.strip() or res.stderr.strip()):
        print(res.stdout + res.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, extra: list[str] | None = None) -> Path:
    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as pool:
        objs = list(pool.map(lambda s: compile_one(s, verbose, extra), srcs))
    if not LIB.exists() or extra or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    args = sys.argv[1:]
    print(build(verbose="-v" in args, extra=["-Xptxas", "-v"] if "--ptxas" in args else None))
