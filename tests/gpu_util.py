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


def bf16_step(x):
    """One bf16 step at the binade of |x|."""
    return np.ldexp(1.0, np.floor(np.log2(np.abs(x) + 1e-30)).astype(int) - 7)


def assert_hidden_close(actual, expected, operand_scale, max_flip_fraction=0.01):
    """North-star tolerance (rel 2e-2 / abs 1e-3) with one allowance: the
    reference rounds to bf16 at fixed points (each bf16_matvec output, the
    slot mix, mixed + shared); FP32-vs-FP64 accumulation moves a value across
    a rounding midpoint now and then, and where addends cancel that one-step
    flip of an operand (size `operand_scale`) lands in a small output. Such
    elements may differ by up to two bf16 steps of the operand scale, and
    must be rare."""
    err = np.abs(actual - expected)
    strict = 1e-3 + 2e-2 * np.abs(expected)
    loose = strict + 2 * bf16_step(operand_scale)
    bad = np.nonzero(err > loose)
    assert bad[0].size == 0, (f"{bad[0].size} elements beyond tolerance; first {[b[:3] for b in bad]}: "
                              f"got {actual[bad][:3]} want {expected[bad][:3]}")
    assert (err > strict).mean() <= max_flip_fraction, f"{(err > strict).mean():.4f} of elements need the allowance"
