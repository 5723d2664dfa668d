"""Compiles and runs tests/cpp/felix_api_test.cpp against libfelix_b200.so: the
C++ operator API (registry, dispatch, exceptions, status) as C++ callers use it;
on a GPU it also computes through every registered reference kernel name and
compares the results with the fp64 oracle."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


@pytest.fixture(scope="module")
def binary(tmp_path_factory):
    import oracle
    oracle.build()  # the GPU mode compares every named kernel with the fp64 oracle
    out = str(tmp_path_factory.mktemp("cpp") / "felix_api_test")
    cmd = ["g++", "-std=c++20", "-O1", os.path.join(ROOT, "tests", "cpp", "felix_api_test.cpp"),
           f"-I{ROOT}/include", f"-I{CUDA}/include", f"-L{ROOT}/sion_b200", "-lfelix_b200",
           f"-Wl,-rpath,{ROOT}/sion_b200", f"-L{ROOT}/oracle", "-loracle",
           f"-Wl,-rpath,{ROOT}/oracle", f"-L{CUDA}/lib64", "-lcudart", "-o", out]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


def _run(binary, *args):
    r = subprocess.run([binary, *args], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all checks passed" in r.stdout


def test_felix_cpp_api_cpu(binary):
    import torch
    if torch.cuda.is_available():
        pytest.skip("covered by the GPU variant")
    _run(binary)


@pytest.mark.gpu
def test_felix_cpp_api_gpu(binary):
    _run(binary, "gpu")
