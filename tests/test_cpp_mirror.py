"""The C++17 host mirror (include/sdq.hpp): tests/cpp/test_sdq_hpp.cpp restates the
reference's quantised-weight tests through it.  On CPU the program must build against the
header and link against libsdq; on a GPU it must run with every check passing."""
from __future__ import annotations

import os
import shutil
import subprocess

import pytest

from conftest import gpu_available

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "stable-diffusion.rs_b200")
CUDA = "/usr/local/cuda"


def _build(out_dir) -> str:
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    exe = os.path.join(str(out_dir), "test_sdq_hpp")
    cmd = [cxx, "-std=c++17", "-O1", "-Wall", "-Wno-unused-function",
           "-I", os.path.join(ROOT, "include"), "-I", os.path.join(CUDA, "include"),
           os.path.join(ROOT, "tests", "cpp", "test_sdq_hpp.cpp"), "-o", exe,
           "-L", PKG, "-lsdq", f"-Wl,-rpath,{PKG}", "-L", os.path.join(CUDA, "lib64"), "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


def test_cpp_mirror_builds_and_links(tmp_path):
    _build(tmp_path)


@pytest.mark.gpu
@pytest.mark.skipif(not gpu_available(), reason="needs an sm_100 device")
def test_cpp_mirror_runs_the_reference_checks(tmp_path):
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 failure(s)" in r.stdout
    assert r.stdout.count("ok  ") == 7
