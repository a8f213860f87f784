"""The drop-in boundary from a C host: include/klearu_gpu.h compiles as
strict C99 (and C++17), a C program links libklearu_gpu.so, and the
host-only entry points (ABI version, argument errors, the LibSVM parser and
the batch iterator) behave as the reference's tests for them say.  No GPU."""

import shutil
import subprocess
from pathlib import Path

import pytest

from klearu_b200 import _lib

ROOT = Path(__file__).resolve().parent.parent


def _cc(name):
    exe = shutil.which(name)
    if not exe:
        pytest.skip(f"{name} not found")
    return exe


def test_c99_host_program(tmp_path):
    cc = _cc("gcc")
    exe = tmp_path / "abi_host"
    libdir = str(_lib.LIB_PATH.parent)
    subprocess.run([cc, "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "native" / "abi_host.c"), "-o", str(exe), "-L", libdir,
                    "-l:libklearu_gpu.so", "-Wl,-rpath," + libdir], check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert res.returncode == 0, res.stderr
    assert res.stdout.strip() == "ok"


def test_header_compiles_as_cpp(tmp_path):
    cxx = _cc("g++")
    src = tmp_path / "t.cpp"
    src.write_text('#include "klearu_gpu.h"\nint main() { return kl_abi_version() == KLEARU_GPU_ABI_VERSION ? 0 : 1; }\n')
    subprocess.run([cxx, "-std=c++17", "-Wall", "-Wextra", "-pedantic", "-Werror", "-fsyntax-only", "-I",
                    str(ROOT / "include"), str(src)], check=True)
