"""Build the native libraries in-tree.

* ``klearu_b200/libklearu_gpu.so`` -- the CUDA engine (sm_100a) behind
  ``include/klearu_gpu.h``, compiled by nvcc from ``klearu_b200/csrc``.
* ``oracle/liboracle.so`` -- the CPU parity checker and CPU baseline, compiled
  by g++ from ``oracle/oracle.cpp`` (see ``oracle/build.py``).

Run ``python -m klearu_b200.build`` from the repository root.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "klearu_b200"
CSRC = PKG / "csrc"
BUILD = ROOT / "_build" / "gpu"
LIB = PKG / "libklearu_gpu.so"
SOURCES = ["hash.cu", "hash_tc.cu", "index.cu", "layer.cu", "shard.cu", "dejavu.cu", "data.cu", "api.cu"]

def _nccl_dirs() -> tuple[str, str]:
    """NCCL headers and library: the copy PyTorch itself loads (nvidia-nccl
    wheel), so one process never holds two NCCL builds."""
    try:
        import nvidia.nccl as _n  # noqa: PLC0415

        base = Path(list(_n.__path__)[0])
        if (base / "include" / "nccl.h").exists() and (base / "lib" / "libnccl.so.2").exists():
            return str(base / "include"), str(base / "lib")
    except ImportError:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


NCCL_INC, NCCL_LIB = _nccl_dirs()

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(ROOT / "include"), "-I", NCCL_INC,
]


def _nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_gpu(verbose: bool = False, force: bool = False) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    nvcc = _nvcc()
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [ROOT / "include" / "klearu_gpu.h"]
    objs = []
    jobs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (Path(src).stem + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            jobs.append([nvcc, *NVCC_FLAGS, "-c", str(s), "-o", str(o)])
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        for cmd, res in zip(jobs, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
            if verbose or res.returncode:
                sys.stderr.write(res.stdout + res.stderr)
            if res.returncode:
                raise RuntimeError("nvcc failed: " + " ".join(cmd))
    if force or _stale(LIB, objs):
        cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(LIB),
               *map(str, objs), "-lcudart", "-L", NCCL_LIB, "-l:libnccl.so.2",
               "-Xlinker", "-rpath=" + NCCL_LIB]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link failed")
    return LIB


def build_all(verbose: bool = False, force: bool = False) -> None:
    build_gpu(verbose=verbose, force=force)
    sys.path.insert(0, str(ROOT))
    from oracle.build import build_oracle  # noqa: E402  (test infrastructure)

    build_oracle(force=force)


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
