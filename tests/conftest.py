"""Shared pytest configuration: markers and import paths.

`gpu` tests need a B200 and the built CUDA library; everything else runs on
the CPU (oracle pins, host logic, C-ABI export checks, gloo multi-rank logic).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "project-k3x_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 device and the built k3xb library")
    config.addinivalue_line("markers", "slow: longer CPU test")


@pytest.fixture(scope="session")
def rs():
    from oracle import Restatement
    return Restatement()


@pytest.fixture(scope="session")
def ref():
    from oracle import Reference, have_reference
    if not have_reference():
        pytest.skip("oracle/_ref/libk3x_ref.so not built (reference tree absent)")
    return Reference()


# GPU files in dependency order: the kernels first, then what is composed of
# them or added on top (golden end-to-end cases, the routing policy, expert
# parallelism, LatentMoE, the device drafter, the host-I/O entry points,
# resident weights, phase timing, expert-parallel failure detection, the
# reference's own layer drivers over the adapter, the block attention
# residual of the token graph), so that a run which stops at the first failure
# stops at the lowest broken layer. Files not listed keep their place after
# these; test_zz_no_alloc.py stays last.
_GPU_ORDER = ["test_gpu_synth", "test_gpu_parity", "test_gpu_mxf4", "test_gpu_linear", "test_gpu_layer", "test_gpu_golden", "test_gpu_c4_oracle",
              "test_gpu_routing_policy", "test_gpu_ep", "test_gpu_ep_verify", "test_gpu_latent", "test_gpu_draft", "test_gpu_host_io",
              "test_gpu_resident", "test_gpu_profile", "test_gpu_ep_failure", "test_gpu_reference_drivers",
              "test_gpu_attnres"]


def pytest_collection_modifyitems(session, config, items):
    def rank(item):
        name = item.module.__name__.rsplit(".", 1)[-1] if item.module else ""
        if name.startswith("test_zz"):
            return len(_GPU_ORDER) + 1
        return _GPU_ORDER.index(name) if name in _GPU_ORDER else len(_GPU_ORDER)
    items.sort(key=rank)   # stable: order inside a file is kept
