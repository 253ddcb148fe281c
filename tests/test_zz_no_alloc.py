"""k3xb_route_static: routing without any device allocation.

For callers that must not allocate device memory mid-run (a serving loop
that reserved all of HBM, a foreign allocator owning the device, or a loop
where cudaMalloc's implicit synchronisation is unacceptable). The entry
point keeps its logits in a fixed 1 MiB array inside the library. This file
is collected last on purpose, so a run that stops at the first failure has
already run every other test; it also passes on its own in a fresh process.
"""
import ctypes as C

import numpy as np
import pytest

from gpu_util import to_dev, torch_cuda
from oracle import bf16_normal, bf16_words

pytestmark = pytest.mark.gpu


def _static_fn():
    import k3xb
    fn = k3xb.library().k3xb_route_static
    vp, u32 = C.c_void_p, C.c_uint32
    fn.argtypes = [vp, u32, u32, vp, vp, u32, u32, vp, vp, vp, vp]
    fn.restype = C.c_int
    return fn


def _dev_ptr(t):
    return C.c_void_p(t.data_ptr())


def test_route_static_matches_route_on_two_calls():
    torch = torch_cuda()
    import k3xb
    ctx = k3xb.Context(0)
    ctx.use_stream()
    fn = _static_fn()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = np.random.default_rng(2026)
    T, H, E, K = 64, 7168, 384, 16
    router = to_dev(torch, bf16_words(g.normal(0, 0.02, size=(E, H))))
    corr = to_dev(torch, g.normal(0, 0.02, size=E).astype(np.float32))
    for call in range(2):   # two calls in a row share (and reuse) the static array
        hidden = to_dev(torch, bf16_normal(g, (T, H)))
        ids_ref = torch.empty((T, K), dtype=torch.int32, device="cuda")
        con_ref = torch.empty((T, K), dtype=torch.float32, device="cuda")
        ctx.route(hidden, router, corr, K, ids_ref, con_ref)
        ids = torch.full((T, K), -1, dtype=torch.int32, device="cuda")
        con = torch.zeros((T, K), dtype=torch.float32, device="cuda")
        status = torch.full((1,), 99, dtype=torch.int32, device="cuda")
        st = fn(_dev_ptr(hidden), T, H, _dev_ptr(router), _dev_ptr(corr), E, K, _dev_ptr(ids), _dev_ptr(con),
                _dev_ptr(status), stream)
        assert st == k3xb.OK, f"call {call}: status {st}"
        torch.cuda.synchronize()
        ctx.sync()
        assert int(status.item()) == 0
        np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy())
        np.testing.assert_allclose(con.cpu().numpy(), con_ref.cpu().numpy(), rtol=1e-6, atol=0)
    ctx.close()


def test_route_static_allocates_nothing_and_runs_without_status():
    """A warm call changes no device memory reservation (cudaMemGetInfo's
    free bytes are the same before and after it), and a call with status
    NULL gives the same routes as k3xb_route."""
    torch = torch_cuda()
    import k3xb
    ctx = k3xb.Context(0)
    ctx.use_stream()
    fn = _static_fn()
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    g = np.random.default_rng(2027)
    T, H, E, K = 32, 7168, 384, 16
    router = to_dev(torch, bf16_words(g.normal(0, 0.02, size=(E, H))))
    corr = to_dev(torch, g.normal(0, 0.02, size=E).astype(np.float32))
    hidden = to_dev(torch, bf16_normal(g, (T, H)))
    ids_ref = torch.empty((T, K), dtype=torch.int32, device="cuda")
    con_ref = torch.empty((T, K), dtype=torch.float32, device="cuda")
    ctx.route(hidden, router, corr, K, ids_ref, con_ref)
    ctx.sync()
    ids = torch.full((T, K), -1, dtype=torch.int32, device="cuda")
    con = torch.zeros((T, K), dtype=torch.float32, device="cuda")
    args = (_dev_ptr(hidden), T, H, _dev_ptr(router), _dev_ptr(corr), E, K, _dev_ptr(ids), _dev_ptr(con), None,
            stream)
    assert fn(*args) == k3xb.OK   # the first call on the device does its one-time set-up
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        assert fn(*args) == k3xb.OK
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device free memory moved by {free0 - free1} bytes"
    np.testing.assert_array_equal(ids.cpu().numpy(), ids_ref.cpu().numpy())
    np.testing.assert_allclose(con.cpu().numpy(), con_ref.cpu().numpy(), rtol=1e-6, atol=0)
    ctx.close()


def test_route_static_rejects_oversize():
    torch = torch_cuda()
    import k3xb
    fn = _static_fn()
    T, H, E, K = 1024, 64, 384, 4    # 393216 logits > 262144
    hidden = torch.zeros((T, H), dtype=torch.float32, device="cuda")
    router = torch.zeros((E, H), dtype=torch.int16, device="cuda")
    corr = torch.zeros(E, dtype=torch.float32, device="cuda")
    ids = torch.zeros((T, K), dtype=torch.int32, device="cuda")
    con = torch.zeros((T, K), dtype=torch.float32, device="cuda")
    st = fn(_dev_ptr(hidden), T, H, _dev_ptr(router), _dev_ptr(corr), E, K, _dev_ptr(ids), _dev_ptr(con),
            None, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == k3xb.INVALID_EXTENT
