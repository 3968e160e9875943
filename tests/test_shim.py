"""The C++ shim (include/gsv_kern_cuda.hpp) with the reference's signatures:
compiles here; its restated test_accel.cpp cases run on the GPU."""
import os
import subprocess

import pytest

from conftest import ROOT

CUDA = "/usr/local/cuda"


def _compile(tmp_path, syntax_only):
    src = os.path.join(ROOT, "tests", "cpp", "shim_test.cpp")
    pkg = os.path.join(ROOT, "gpt-sovits-native_b200")
    cmd = ["g++", "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(CUDA, "include"), src]
    if syntax_only:
        cmd += ["-fsyntax-only"]
    else:
        exe = str(tmp_path / "shim_test")
        cmd += ["-o", exe, "-L", pkg, "-lgsvk", f"-Wl,-rpath,{pkg}",
                "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{CUDA}/lib64"]
    subprocess.run(cmd, check=True)
    return None if syntax_only else exe


def test_shim_header_compiles(tmp_path):
    _compile(tmp_path, syntax_only=True)


@pytest.mark.gpu
def test_shim_cases_on_device(tmp_path):
    exe = _compile(tmp_path, syntax_only=False)
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "PASS" in out.stdout
