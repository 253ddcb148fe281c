"""The C++20 host layer (include/k3xb.hpp) compiles with -Wall -Wextra
-Werror against the C ABI, links libk3xb.so, and behaves on the host:
verification unpacking, the drafting round, and context creation that
fails with a status (no fallback) when there is no B200."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "project-k3x_b200", "k3xb")


def test_cpp_adapter(tmp_path):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no C++ compiler")
    if not os.path.exists(os.path.join(LIBDIR, "libk3xb.so")):
        pytest.fail("libk3xb.so is not built (project-k3x_b200/build.py)")
    exe = tmp_path / "adapter_check"
    subprocess.run([cxx, "-std=c++20", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "adapter_check.cpp"), "-L", LIBDIR, "-lk3xb",
                    f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert out.stdout.startswith("adapter ok"), out.stdout
