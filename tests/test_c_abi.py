"""The C ABI from C: tests/c_abi/abi_check.c is compiled by a plain C compiler
against include/int4kv_b200.h and linked to libint4kv_b200.so -- the way a C,
cgo or FFI host of the reference's launchers binds the library -- and run.
It exercises only host-side argument checks, so no GPU is needed."""

import os
import shutil
import subprocess

import pytest

from helpers import pkg

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cuda_include():
    for cand in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if cand and os.path.exists(os.path.join(cand, "include", "cuda_runtime.h")):
            return os.path.join(cand, "include")
    return None


def test_c_host_links_and_gets_documented_answers(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    inc = _cuda_include()
    if not cc or not inc:
        pytest.skip("no C compiler or CUDA headers")
    lib = pkg("_build").build()
    exe = str(tmp_path / "abi_check")
    cmd = [cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), "-I", inc,
           os.path.join(ROOT, "tests", "c_abi", "abi_check.c"), lib,
           "-Wl,-rpath," + os.path.dirname(lib), "-o", exe]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stderr
    run = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert "c abi ok" in run.stdout
