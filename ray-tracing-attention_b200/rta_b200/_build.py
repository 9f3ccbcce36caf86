"""Build librta_cuda.so (sm_100a) and the rta_worker executable in-tree.

nvcc cross-compiles for sm_100a without a GPU, so this runs on the CPU build
host and again, if sources are newer than the binary, on a GPU box.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = ROOT / "csrc"
WORKER_SRC = ROOT / "worker"
INCLUDE = ROOT.parent / "include"
OBJ = ROOT.parent / "_build" / "rta"
LIBRARY = PKG / "librta_cuda.so"
WORKER = PKG / "rta_worker"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: librta_cuda.so cannot be built (the CUDA path has no fallback)")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    srcs = _sources()
    if not force and not _stale(LIBRARY, srcs + _headers()):
        return LIBRARY
    OBJ.mkdir(parents=True, exist_ok=True)
    cc = nvcc()

    def compile_one(src: Path) -> Path:
        obj = OBJ / (src.stem + ".o")
        if force or _stale(obj, [src] + _headers()):
            cmd = [cc, *NVCC_FLAGS, *ARCH, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode:
                raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
            if verbose and r.stderr.strip():
                print(r.stderr)
        return obj

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as pool:
        objs = list(pool.map(compile_one, srcs))
    tmp = LIBRARY.with_suffix(f".{os.getpid()}.tmp")
    r = subprocess.run([cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs)], capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


def build_worker(force: bool = False) -> Path | None:
    src = WORKER_SRC / "rta_worker.cpp"
    if not src.exists():
        return None
    lib = build_library()
    if not force and not _stale(WORKER, [src, lib] + _headers()):
        return WORKER
    tmp = WORKER.with_suffix(f".{os.getpid()}.tmp")
    r = subprocess.run(["g++", "-std=c++17", "-O2", "-I", str(INCLUDE), str(src), "-o", str(tmp),
                        "-L", str(PKG), "-lrta_cuda", "-Wl,-rpath,$ORIGIN"], capture_output=True, text=True)
    if r.returncode:
        raise RuntimeError(f"worker build failed:\n{r.stderr}")
    os.replace(tmp, WORKER)
    return WORKER


def build_all(force: bool = False) -> None:
    build_library(force)
    build_worker(force)


if __name__ == "__main__":
    import sys
    build_all(force="--force" in sys.argv)
    print(LIBRARY)
