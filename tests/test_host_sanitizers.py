"""Host code under AddressSanitizer and UndefinedBehaviorSanitizer: the
resident weight table (csrc/resident.hpp), the expert-parallel bounded
waits (csrc/ep_guard.hpp), the C++20 host layer (include/k3xb.hpp) and the
ComputeBackend adapter, each built from the same
sources as their plain tests with -fsanitize=address,undefined and run to a
clean exit. Device code has no sanitizer here (compute-sanitizer is closed
on the GPU pool); its guards are bounded waits, status words and the
parity tests."""
import os
import shutil
import subprocess

import pytest

from test_backend_adapter import ADAPTER, reference_include

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "project-k3x_b200", "k3xb")
SAN = ["-fsanitize=address,undefined", "-fno-sanitize-recover=all", "-fno-omit-frame-pointer", "-g", "-O1"]


def _run(tmp_path, name, sources, extra, expect, env_extra=None):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no C++ compiler")
    exe = tmp_path / name
    subprocess.run([cxx, "-std=c++20", "-Wall", "-Wextra", "-Werror", *SAN, *extra, *sources, "-o", str(exe)],
                   check=True)
    env = dict(os.environ, UBSAN_OPTIONS="print_stacktrace=1:halt_on_error=1")
    env.update(env_extra or {})
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300, env=env)
    assert out.returncode == 0, out.stderr[-4000:]
    assert out.stdout.startswith(expect), out.stdout
    assert "runtime error" not in out.stderr, out.stderr[-4000:]


def test_resident_table_sanitized(tmp_path):
    _run(tmp_path, "resident_check", [os.path.join(ROOT, "tests", "cpp", "resident_check.cpp")],
         ["-I", os.path.join(ROOT, "include"), "-I", os.path.join(ROOT, "project-k3x_b200", "csrc")],
         "resident ok", {"ASAN_OPTIONS": "detect_leaks=1"})


def test_adapter_protocol_sanitized(tmp_path):
    """The adapter's token and slot bookkeeping under the reference's drivers
    (tests/cpp/adapter_protocol_check.cpp) with leak checking: everything is
    host code there (the C ABI is the scripted stand-in)."""
    from test_backend_adapter import protocol_sources
    inc, sources = protocol_sources()
    if not inc:
        pytest.skip("reference sources absent")
    _run(tmp_path, "adapter_protocol_check", sources, ["-isystem", inc, "-I", os.path.join(ROOT, "include"),
                                                      "-I", ADAPTER], "adapter protocol ok",
         {"ASAN_OPTIONS": "detect_leaks=1"})


def test_ep_guard_sanitized(tmp_path):
    _run(tmp_path, "ep_guard_check", [os.path.join(ROOT, "tests", "cpp", "ep_guard_check.cpp")],
         ["-I", os.path.join(ROOT, "project-k3x_b200", "csrc")], "ep guard ok", {"ASAN_OPTIONS": "detect_leaks=1"})


def _needs_lib():
    if not os.path.exists(os.path.join(LIBDIR, "libk3xb.so")):
        pytest.fail("libk3xb.so is not built (project-k3x_b200/build.py)")


# libk3xb.so (not instrumented) links the CUDA runtime, whose one-time
# allocations are not ours to free: leak checking stays off for these two.
def test_cpp_host_layer_sanitized(tmp_path):
    _needs_lib()
    _run(tmp_path, "adapter_check", [os.path.join(ROOT, "tests", "cpp", "adapter_check.cpp")],
         ["-I", os.path.join(ROOT, "include"), "-L", LIBDIR, "-lk3xb", f"-Wl,-rpath,{LIBDIR}"],
         "adapter ok", {"ASAN_OPTIONS": "detect_leaks=0"})


def test_backend_adapter_sanitized(tmp_path):
    _needs_lib()
    inc = reference_include()
    if not inc:
        pytest.skip("reference headers absent")
    _run(tmp_path, "backend_adapter_check",
         [os.path.join(ADAPTER, "backend_b200.cpp"), os.path.join(ROOT, "tests", "cpp", "backend_adapter_check.cpp")],
         ["-isystem", inc, "-I", os.path.join(ROOT, "include"), "-I", ADAPTER, "-L", LIBDIR, "-lk3xb",
          f"-Wl,-rpath,{LIBDIR}"],
         "backend adapter ok", {"ASAN_OPTIONS": "detect_leaks=0"})
