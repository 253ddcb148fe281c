"""Helpers shared by the GPU parity tests (torch for device memory only)."""
import numpy as np
import pytest


def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("a CUDA device is required for -m gpu tests")
    return torch


def to_dev(torch, a, dtype=None):
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a.view(np.int16) if a.dtype == np.uint16 else a)
    return t.cuda()


def from_dev(t, dtype):
    a = t.cpu().numpy()
    return a.view(dtype) if a.dtype != dtype else a


def layer_to_dev(torch, layer: dict) -> dict:
    out = {}
    for k, v in layer.items():
        out[k] = to_dev(torch, v) if isinstance(v, np.ndarray) else v
    return out


def assert_close_bf16(actual, expected, rtol=2e-2, atol=1e-3):
    """The north-star tolerance for hidden states and logits."""
    np.testing.assert_allclose(actual, expected, rtol=rtol, atol=atol)
