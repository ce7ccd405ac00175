"""Builds libnpl_b200.so in-tree for sm_100a.

Every .cu / .cpp under csrc/ is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a`` (host code through g++), and the
objects are linked into ``<package>/lib/libnpl_b200.so`` with the CUDA runtime
linked statically, so the library does not depend on which libcudart a host
process (for example PyTorch) has already loaded. Rebuilds are incremental on
file modification times.

Usage:  python -m npl_b200.build   (from the package directory)  or  build().
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent.parent  # project-jcore_b200/
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = PKG_DIR / "_build"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libnpl_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC,-fvisibility=hidden",
    "-Xptxas",
    "-warn-spills",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
    f"-I{CSRC / 'kernels'}",
    "-DNPL_B200_BUILD",
]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build")
    return cand


def _sources() -> list[Path]:
    return sorted(list(CSRC.rglob("*.cu")) + list(CSRC.rglob("*.cpp")))


def _headers() -> list[Path]:
    hs = list(CSRC.rglob("*.h")) + list(CSRC.rglob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return hs


def _obj_for(src: Path) -> Path:
    rel = src.relative_to(CSRC)
    return BUILD_DIR / (str(rel).replace(os.sep, "__") + ".o")


def _compile(src: Path, newest_header: float, verbose: bool) -> tuple[Path, str]:
    obj = _obj_for(src)
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header):
        return obj, ""
    cmd = [_nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [_nvcc(), *NVCC_FLAGS, "-x", "cu", "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    return obj, (res.stderr if verbose else "")


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compiles and links libnpl_b200.so; returns its path."""
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    srcs = _sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: _compile(s, newest_header, verbose), srcs))
    objs = [o for o, _ in results]
    for _, log in results:
        if log:
            sys.stderr.write(log)
    newest_obj = max(o.stat().st_mtime for o in objs)
    if LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= newest_obj:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp),
           *[str(o) for o in objs], "-Xlinker", "--no-undefined", "-lpthread", "-ldl", "-lrt"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
