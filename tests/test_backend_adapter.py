"""B200Backend, the k3x::ComputeBackend over libk3xb
(project-k3x_b200/adapter/), compiled against the reference's own
interface headers with -Wall -Wextra -Werror and linked with libk3xb.so:
the proof that it is a drop-in for backend.hpp:326-462. Its host-side
behaviour (method split, argument checks, statuses, no retry on the other
backend) runs here; its device calls are the C ABI entry points the GPU
tests cover (test_gpu_host_io.py, test_gpu_resident.py).

The reference tree is K3X_REFERENCE when set, else a checkout named
`reference` beside this repository (as in oracle/Makefile); without it the
test skips."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "project-k3x_b200", "k3xb")
ADAPTER = os.path.join(ROOT, "project-k3x_b200", "adapter")


def reference_root():
    return os.environ.get("K3X_REFERENCE") or os.path.abspath(os.path.join(ROOT, "..", "reference"))


def reference_include():
    inc = os.path.join(reference_root(), "runtime", "include")
    return inc if os.path.exists(os.path.join(inc, "k3x", "backend.hpp")) else None


def test_backend_adapter_against_reference_interface(tmp_path):
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no C++ compiler")
    inc = reference_include()
    if not inc:
        pytest.skip("reference headers absent")
    if not os.path.exists(os.path.join(LIBDIR, "libk3xb.so")):
        pytest.fail("libk3xb.so is not built (project-k3x_b200/build.py)")
    exe = tmp_path / "backend_adapter_check"
    subprocess.run([cxx, "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-isystem", inc,
                    "-I", os.path.join(ROOT, "include"), "-I", ADAPTER,
                    os.path.join(ADAPTER, "backend_b200.cpp"),
                    os.path.join(ROOT, "tests", "cpp", "backend_adapter_check.cpp"),
                    "-L", LIBDIR, "-lk3xb", f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert out.stdout.startswith("backend adapter ok"), out.stdout


def test_reference_layer_driver_harness_loads_and_reports_no_gpu():
    """oracle/_ref/libk3x_ref_b200.so (the reference's official_layer_cuda
    over B200Backend) resolves every symbol, marshals a real layer, and
    without a B200 ends in make_b200_backend's status, BACKEND_UNAVAILABLE
    (the GPU test runs it to completion)."""
    import numpy as np
    import torch

    import golden_util as gu
    from oracle import OracleError, ReferenceOnB200, have_reference_on_b200
    if not have_reference_on_b200():
        if reference_include():
            pytest.fail("oracle/_ref/libk3x_ref_b200.so is not built (make -C oracle after libk3xb.so)")
        pytest.skip("reference tree absent and no prebuilt harness")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present: tests/test_gpu_latent.py runs the harness")
    layer, f = gu.official_layer()
    with pytest.raises(OracleError) as e:
        ReferenceOnB200().official_layer(layer, f["hidden"], f["block"], (f["conv_q"], f["conv_k"], f["conv_v"]),
                                         f["recurrent"])
    assert e.value.status == 17, str(e.value)
    assert np.isfinite(f["hidden"]).all()
    with pytest.raises(OracleError) as e:
        ReferenceOnB200().official_two_layer([layer, layer], f["hidden"][:2], f["block"][:2],
                                             [(f["conv_q"], f["conv_k"], f["conv_v"])] * 2, [f["recurrent"]] * 2)
    assert e.value.status == 17, str(e.value)


def protocol_sources():
    """The adapter protocol check's sources: the check, the scripted C ABI, the
    adapter, and the reference's drivers and the CPU steps they call."""
    inc = reference_include()
    if not inc:
        return None, None
    src = os.path.join(os.path.dirname(inc), "src")
    ref = [os.path.join(src, f) for f in ("official_layer.cpp", "official_two_layer.cpp", "official_moe.cpp",
                                          "official_kda.cpp", "ops.cpp", "profile.cpp")]
    ours = [os.path.join(ROOT, "tests", "cpp", "adapter_protocol_check.cpp"),
            os.path.join(ROOT, "tests", "cpp", "fake_k3xb.cpp"), os.path.join(ADAPTER, "backend_b200.cpp")]
    return inc, ours + ref


def test_adapter_keeps_the_reference_drivers_protocol(tmp_path):
    """The reference's official_layer_cuda (host and device route
    preparation, KDA state seeded then published across calls) and
    official_two_layer_cuda (host_round_trip, device_closure), unchanged,
    over B200Backend with a scripted C ABI (tests/cpp/fake_k3xb.cpp): every
    token, publication flag and output size the drivers check is right, and
    nothing leaks from one run into the next."""
    cxx = shutil.which("g++")
    if not cxx:
        pytest.skip("no C++ compiler")
    inc, sources = protocol_sources()
    if not inc:
        pytest.skip("reference sources absent")
    exe = tmp_path / "adapter_protocol_check"
    subprocess.run([cxx, "-std=c++20", "-O1", "-Wall", "-Wextra", "-Werror", "-isystem", inc,
                    "-I", os.path.join(ROOT, "include"), "-I", ADAPTER, *sources, "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert out.stdout.startswith("adapter protocol ok"), out.stdout
