"""The secondary boundary: libmfb.so as a MatrixProPluginV1 backend of the reference's
BackendRegistry::load_plugin (src/hw/backend_registry.cpp:252-266).

CPU tier: the entry point is exported and returns a version-1 CUDA table; where the
reference's headers are present (the build container), a compile-only check pins the
member offsets of mfb_plugin_v1 / mfb_plugin_gemm_args to MatrixProPluginV1 /
PluginGemmArgs (include/matrix_pro/core/backend_registry.hpp:60-94). GPU tier: a C++ host
loads the library by dlopen and runs a GEMM through the table."""
import ctypes
import os
import subprocess

import pytest

import matrixflash_pro_b200 as mf

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFERENCE_INCLUDE = "/root/reference/include"


class _Table(ctypes.Structure):
    _fields_ = [("abi", ctypes.c_uint32), ("device_type", ctypes.c_int), ("name", ctypes.c_char_p),
                ("user", ctypes.c_void_p)] + [(f, ctypes.c_void_p) for f in (
                    "destroy", "device_count", "device_name", "memory_bytes", "allocate", "deallocate", "copy",
                    "gemm")]


def test_create_returns_a_version_1_cuda_table():
    lib = ctypes.CDLL(mf.LIB_PATH)
    lib.CreateMatrixProBackend.restype = ctypes.POINTER(_Table)
    t = lib.CreateMatrixProBackend().contents
    assert t.abi == 1 and t.device_type == 1 and t.name == b"b200-tcgen05"
    assert all(getattr(t, f) for f in ("destroy", "device_count", "device_name", "memory_bytes", "allocate",
                                       "deallocate", "copy", "gemm"))


@pytest.mark.skipif(not os.path.isdir(REFERENCE_INCLUDE), reason="reference headers not present")
def test_layout_matches_the_reference_plugin_abi(tmp_path):
    src = tmp_path / "layout.cpp"
    fields = ["abi", "device_type", "name", "user", "destroy", "device_count", "device_name", "memory_bytes",
              "allocate", "deallocate", "copy", "gemm"]
    args = ["device", "m", "n", "k", "a", "lda", "b", "ldb", "c", "ldc", "alpha", "beta"]
    lines = ['#include "matrix_pro/core/backend_registry.hpp"', '#include "mfb_plugin.h"', "#include <cstddef>",
             "using R = matrix_pro::MatrixProPluginV1;", "using G = matrix_pro::PluginGemmArgs;",
             "static_assert(sizeof(R) == sizeof(mfb_plugin_v1), \"table size\");",
             "static_assert(sizeof(G) == sizeof(mfb_plugin_gemm_args), \"args size\");"]
    lines += [f"static_assert(offsetof(R, {f}) == offsetof(mfb_plugin_v1, {f}), \"{f}\");" for f in fields]
    lines += [f"static_assert(offsetof(G, {f}) == offsetof(mfb_plugin_gemm_args, {f}), \"{f}\");" for f in args]
    src.write_text("\n".join(lines) + "\n")
    subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-I", REFERENCE_INCLUDE, "-I", os.path.join(ROOT, "include"),
                    str(src)], check=True)


def build_host(tmp_path) -> str:
    exe = str(tmp_path / "plugin_host")
    subprocess.run(["g++", "-std=c++17", "-O2", os.path.join(ROOT, "tests", "cpp", "plugin_host.cpp"),
                    "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
                    "-L", "/usr/local/cuda/lib64", "-lcudart", "-ldl", "-Wl,-rpath,/usr/local/cuda/lib64",
                    "-o", exe], check=True)
    return exe


def test_plugin_host_compiles(tmp_path):
    assert os.path.exists(build_host(tmp_path))


@pytest.mark.gpu
def test_plugin_gemm_through_the_table(tmp_path):
    exe = build_host(tmp_path)
    out = subprocess.run([exe, mf.LIB_PATH], capture_output=True, text=True, timeout=120)
    print(out.stdout)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "0 failure(s)" in out.stdout
