"""Failure detection of the expert-parallel path on the GPU, without a
GPU fault: the bounded-wait surface on a healthy world of one (nonblocking
communicator, status, finalize), and two ranks where one leaves between
steps and the other finds it on the host, aborts, and re-forms as a world
of one (needs two GPUs, NVLS off). The scripted-communicator and CPU-rank
cases are in test_ep_failure.py. Ordered after the other GPU files: these
run code paths the validated layers do not need.
"""
import os

import numpy as np
import pytest

from gpu_util import torch_cuda
from oracle import bf16_normal
from test_gpu_ep import DIMS, _ep, _layer, _one_gpu

pytestmark = pytest.mark.gpu

def test_ep_failure_detection_surface_on_a_healthy_world_of_one(rs):
    """Status before init is INVALID_STATE; a nonblocking communicator
    (creation and each exchange's launch settled under the bound) gives the
    blocking one's bits; status stays OK across calls; finalize drains.
    A failing peer is exercised on the CPU (test_ep_failure.py)."""
    import k3xb
    torch = torch_cuda()
    layer = _layer(rs)
    x = bf16_normal(np.random.default_rng(60), (12, DIMS["hidden"]))
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        with pytest.raises(k3xb.K3xbError) as e:
            ctx.ep_status()
        assert e.value.status == k3xb.INVALID_STATE
        want = _one_gpu(torch, ctx, layer, x)
        ctx.ep_init(k3xb.ep_unique_id(), 0, 1, timeout_ms=60000, nonblocking=True)
        ctx.ep_status()
        for _ in range(2):
            got = _ep(torch, ctx, layer, x, 0, 1)
            for g, w in zip(got, want):
                np.testing.assert_array_equal(g, w)
            ctx.ep_status()
        ctx.ep_finalize()
        with pytest.raises(k3xb.K3xbError):
            ctx.ep_status()
    finally:
        ctx.close()


def _departing_rank_main(rank, world, uid, port, out_dir):
    """Step 0 on both ranks; then rank 1 leaves between steps. Rank 0 learns
    it on the host before its next launch (no collective is ever left in
    flight), aborts, and goes on as a world of one."""
    import sys
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "project-k3x_b200"), os.path.join(root, "oracle")]
    import torch

    import k3xb
    from k3xb.peers import PeerLost, PeerWatch, make_store
    from oracle import Restatement
    torch.cuda.set_device(rank)
    store = make_store(rank, world, port=port, timeout_s=60)
    watch = PeerWatch(store, rank, world, timeout_s=60)
    rs = Restatement()
    layer = _layer(rs)
    x = bf16_normal(np.random.default_rng(61), (8 * world, DIMS["hidden"]))
    ctx = k3xb.Context(rank)
    ctx.use_stream()
    ctx.ep_init(uid, rank, world, timeout_ms=60000)
    watch.step(0)
    out0, _, _ = _ep(torch, ctx, layer, x, rank, world)   # synchronised: nothing in flight after it
    if rank == 1:
        watch.leave()
        store.wait(["test/ack"], __import__("datetime").timedelta(seconds=60))   # rank 0 has synchronised too
        ctx.ep_abort()
        ctx.ep_finalize()
        ctx.close()
        open(os.path.join(out_dir, "r1.txt"), "w").write("left")
        return
    try:
        watch.step(1)
        result = "no loss seen"
    except PeerLost as e:
        result = f"lost {e.missing} departed {e.departed}"
    store.set("test/ack", b"1")
    ctx.ep_abort()
    ctx.ep_finalize()
    ctx.ep_init(k3xb.ep_unique_id(), 0, 1, timeout_ms=60000)   # the survivors re-form
    out1, _, _ = _ep(torch, ctx, layer, x, 0, 1)
    ctx.ep_finalize()
    ctx.close()
    np.save(os.path.join(out_dir, "out0.npy"), out0)
    np.save(os.path.join(out_dir, "out1.npy"), out1)
    open(os.path.join(out_dir, "r0.txt"), "w").write(result)
    import time
    time.sleep(0.5)   # the store's server outlives rank 1's last use of it


def test_ep_departed_rank_found_on_the_host(rs, tmp_path):
    torch = torch_cuda()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import socket

    import torch.multiprocessing as mp

    import k3xb
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    world = 2
    uid = k3xb.ep_unique_id()
    mp.start_processes(_departing_rank_main, args=(world, uid, port, str(tmp_path)), nprocs=world,
                       start_method="spawn")
    assert open(tmp_path / "r1.txt").read() == "left"
    assert open(tmp_path / "r0.txt").read() == "lost [1] departed [1]"
    layer = _layer(rs)
    x = bf16_normal(np.random.default_rng(61), (8 * world, DIMS["hidden"]))
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        want, _, _ = _one_gpu(torch, ctx, layer, x)
    finally:
        ctx.close()
    np.testing.assert_array_equal(np.load(tmp_path / "out0.npy"), want[:8])
    np.testing.assert_array_equal(np.load(tmp_path / "out1.npy"), want)
