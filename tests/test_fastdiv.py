"""CPU tier: the multiply-shift division used by the conv TMA producers (csrc/fastdiv.h).

The conv kernels turn K-block indices into box coordinates with it; a wrong quotient would
read the wrong tap, channel or image. tests/cpp/fastdiv_check.cpp compares it with the
hardware division over the operand range the kernels allow."""
import os
import subprocess

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_fastdiv_matches_division(tmp_path):
    exe = str(tmp_path / "fastdiv_check")
    subprocess.run(["g++", "-std=c++17", "-O2", os.path.join(ROOT, "tests", "cpp", "fastdiv_check.cpp"),
                    "-I", os.path.join(ROOT, "matrixflash_pro_b200", "csrc"), "-o", exe], check=True)
    out = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stdout + out.stderr
    assert " 0 failure(s)" in out.stdout
