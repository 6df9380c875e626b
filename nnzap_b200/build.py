"""Build the in-tree CUDA library ``nnzap_b200/_lib/libnnz_b200.so``.

sm_100a only: ``nvcc -gencode arch=compute_100a,code=sm_100a``.  Each
translation unit compiles in parallel; the result is linked as one shared
library with the CUDA runtime linked statically, so the .so has no torch
dependency and exports only the C ABI of ``include/nnz_b200.h``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libnnz_b200.so"
BUILD = ROOT / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++20", "-lineinfo", "-Xcompiler", "-fPIC,-O3",
              "--expt-relaxed-constexpr", "-I", str(ROOT / "include"), "-I", str(CSRC)]


def _nccl_include() -> list[str]:
    """nccl.h for the run-time-loaded NCCL (types only; the library is dlopen()ed)."""
    try:
        import nvidia.nccl as nn  # the NCCL wheel torch ships with
        inc = Path(list(nn.__path__)[0]) / "include"
        if (inc / "nccl.h").exists():
            return ["-I", str(inc)]
    except ImportError:
        pass
    return []


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the nnzap_b200 CUDA library cannot be built")


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [ROOT / "include" / "nnz_b200.h"]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps)


def build(verbose: bool = False, force: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    OUT_DIR.mkdir(exist_ok=True)
    objs, jobs = [], []
    for src in sources():
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        if force or _stale(obj, src):
            if src.suffix == ".cpp":
                cmd = ["g++", "-O3", "-std=c++20", "-fPIC", "-pthread", "-I", str(CSRC),
                       "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
            else:
                extra = os.environ.get("NNZ_NVCC_EXTRA", "").split()   # experiments only
                cmd = [nvcc, *ARCH, *NVCC_FLAGS, *extra, *_nccl_include(), "-c", str(src), "-o", str(obj)]
            jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=max(1, os.cpu_count() or 1)) as ex:
        for cmd, res in zip(jobs, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
            if verbose or res.returncode:
                sys.stderr.write(" ".join(cmd) + "\n" + res.stdout + res.stderr)
            if res.returncode:
                raise RuntimeError(f"compile failed: {cmd[-3]}")
    if force or jobs or not LIB.exists():
        link = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-cudart", "static",
                "-o", str(LIB), *map(str, objs), "-lpthread", "-ldl"]
        res = subprocess.run(link, capture_output=True, text=True)
        if res.returncode:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link failed")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
