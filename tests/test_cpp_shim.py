"""Builds the C++ drop-in test (tests/cpp/test_attn_shim.cc) with the host
compiler against include/molot_b200/attn.hpp and the C-ABI library, and runs
it on the GPU.  The build step alone runs without a GPU."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SRC = os.path.join(ROOT, "tests", "cpp", "test_attn_shim.cc")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _build(tmp_path):
    import oracle
    oracle.build(with_ref=False)
    exe = str(tmp_path / "test_attn_shim")
    cxx = os.environ.get("CXX", "g++")
    libdir = os.path.join(ROOT, "molot_b200")
    odir = os.path.join(ROOT, "oracle", "_build")
    cmd = [cxx, "-std=c++17", "-O2", "-I", os.path.join(ROOT, "include"), "-I",
           os.path.join(CUDA, "include"), SRC, "-o", exe,
           "-L", libdir, "-lmolot_b200", f"-Wl,-rpath,{libdir}",
           "-L", odir, "-lmolot_oracle", f"-Wl,-rpath,{odir}",
           "-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{os.path.join(CUDA, 'lib64')}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)
    return exe


def test_cpp_shim_compiles(tmp_path):
    assert os.path.isfile(_build(tmp_path))


@pytest.mark.gpu
def test_cpp_shim_runs(tmp_path, torch_cuda):
    exe = _build(tmp_path)
    r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all checks passed" in r.stdout
