"""The product path never reaches the oracle: the package and the library
neither import, link nor load anything under oracle/ (test infrastructure,
used only by tests/, __graft_entry__.smoke() and bench.py's CPU baseline and
reference arms), and the adapter does not name it."""
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "project-k3x_b200")


def _sources():
    for base, _, files in os.walk(PKG):
        if "_build" in base:
            continue
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".hpp", ".h")):
                yield os.path.join(base, f)


def test_package_and_kernels_do_not_load_the_oracle():
    """No import of the oracle package and no name of its libraries. Comments
    may cite oracle/k3x_oracle.c where it defines a canonical order the
    kernels follow (rejection sampling has no reference counterpart)."""
    bad = []
    for path in _sources():
        text = open(path, encoding="utf-8").read()
        if re.search(r"^\s*(import|from)\s+oracle\b|libk3x_oracle|libk3x_ref|oracle/_ref", text, re.M):
            bad.append(os.path.relpath(path, ROOT))
    assert not bad, bad


def test_library_links_no_oracle():
    lib = os.path.join(PKG, "k3xb", "libk3xb.so")
    if not os.path.exists(lib):
        pytest.fail("libk3xb.so is not built (project-k3x_b200/build.py)")
    needed = subprocess.run(["readelf", "-d", lib], capture_output=True, text=True).stdout
    assert "k3x_oracle" not in needed and "k3x_ref" not in needed, needed
