"""CPU-side checks of the C ABI: the library loads, exports every symbol that
include/k3xb.h declares, and fails loudly (no CPU fallback) without a GPU."""
import ctypes as C
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "k3xb.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*int\s+(k3xb_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_symbols()
    for required in ("k3xb_create", "k3xb_route", "k3xb_expert_major_plan", "k3xb_moe_layer_forward",
                     "k3xb_moe_layer_forward_host", "k3xb_kda_tree", "k3xb_kda_commit",
                     "k3xb_accept_greedy", "k3xb_accept_rejection"):
        assert required in names


def test_library_exports_every_declared_symbol():
    import k3xb
    lib = k3xb.library()
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_no_gpu_fails_loudly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    import k3xb
    with pytest.raises(k3xb.K3xbError) as e:
        k3xb.Context(0)
    assert e.value.status == k3xb.BACKEND_UNAVAILABLE


def test_null_context_rejected():
    import k3xb
    lib = k3xb.library()
    assert lib.k3xb_sync(None) == k3xb.INVALID_EXTENT
    assert lib.k3xb_destroy(None) == k3xb.OK
