"""The resident weight table (project-k3x_b200/csrc/resident.hpp) on the
host: the same source the library runs over device memory, compiled here
against a malloc-backed arena. Checks the reference's rules for
device-resident weights (runtime/cuda/resident_weights.cu:104-166: hit,
admitted, bypass, payload and shape checks, capacity) and the B200
additions (MXFP4 admission validation, tcgen05 scale copies, expert
stacks in the grouped-GEMM layout)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_resident_table_rules(tmp_path):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no C++ compiler")
    exe = tmp_path / "resident_check"
    subprocess.run([cxx, "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror",
                    "-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "project-k3x_b200", "csrc"),
                    os.path.join(ROOT, "tests", "cpp", "resident_check.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert out.stdout.startswith("resident ok"), out.stdout
