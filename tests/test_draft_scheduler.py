"""The draft-length schedule of the C++20 host layer (include/k3xb.hpp,
DraftLengthScheduler) against the reference's AdaptiveDraftScheduler
(runtime/src/aurora_scheduler.cpp, compiled in place from the reference
tree): 120,000 decisions over 400 seeded configurations and outcome
sequences, valid and invalid, must agree in every chosen length, status and
counter. Skips where the reference tree is absent."""
import os
import shutil
import subprocess

import pytest

from test_backend_adapter import reference_include

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_draft_scheduler_matches_reference(tmp_path):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no C++ compiler")
    inc = reference_include()
    if not inc:
        pytest.skip("reference headers absent")
    src = os.path.join(os.path.dirname(inc), "src", "aurora_scheduler.cpp")
    exe = tmp_path / "scheduler_check"
    subprocess.run([cxx, "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-fsanitize=address,undefined",
                    "-fno-sanitize-recover=all", "-isystem", inc, "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "scheduler_check.cpp"), src, "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-4000:]
    assert out.stdout.startswith("scheduler ok 120000"), out.stdout
