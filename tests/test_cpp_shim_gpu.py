"""GPU tier: C++17 reference-side bodies over the C ABI, compiled with g++ against include/mfb.h
and libmfb.so and run as their own processes:

* tests/cpp/cuda_hooks_shim.cpp: matrix_pro::hw::cuda_gemm / cuda_sync;
* tests/cpp/matrix_api_shim.cpp: GemmPlan, gemm_into / gemm with the per-thread plan cache, and
  conv2d, running the reference's known answers (tests/unit/test_gemm_plan.cpp:14-88,
  tests/unit/test_conv.cpp:31-67)."""
import os
import subprocess

import pytest

import matrixflash_pro_b200 as mf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_shim(tmp_path, name="cuda_hooks_shim") -> str:
    exe = str(tmp_path / name)
    libdir = os.path.dirname(mf.LIB_PATH)
    subprocess.run(["g++", "-std=c++17", "-O2", "-Wall", os.path.join(ROOT, "tests", "cpp", f"{name}.cpp"),
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


def test_matrix_api_shim_compiles(tmp_path):
    assert os.path.exists(build_shim(tmp_path, "matrix_api_shim"))


@pytest.mark.gpu
def test_matrix_api_shim_known_answers_on_device(tmp_path):
    exe = build_shim(tmp_path, "matrix_api_shim")
    out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    print(out.stdout)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 failure(s)" in out.stdout
