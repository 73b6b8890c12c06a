"""GPU tier: the C++ drop-in body of matrix_pro::hw::cuda_gemm / cuda_sync over the C ABI,
compiled with g++ against include/mfb.h and libmfb.so and run as its own process."""
import os
import subprocess

import pytest

import matrixflash_pro_b200 as mf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_shim(tmp_path) -> str:
    exe = str(tmp_path / "cuda_hooks_shim")
    libdir = os.path.dirname(mf.LIB_PATH)
    subprocess.run(["g++", "-std=c++17", "-O2", os.path.join(ROOT, "tests", "cpp", "cuda_hooks_shim.cpp"),
                    "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include", "-L", libdir, "-lmfb",
                    "-L", "/usr/local/cuda/lib64", "-lcudart", f"-Wl,-rpath,{libdir}",
                    "-Wl,-rpath,/usr/local/cuda/lib64", "-o", exe], check=True)
    return exe


def test_shim_compiles(tmp_path):
    assert os.path.exists(build_shim(tmp_path))


@pytest.mark.gpu
def test_shim_runs_on_device(tmp_path):
    exe = build_shim(tmp_path)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    print(out.stdout)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "0 failure(s)" in out.stdout
