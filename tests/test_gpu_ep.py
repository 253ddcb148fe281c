"""Expert-parallel MoE layer through the C ABI (k3xb_ep_*): NCCL all-to-all
dispatch / combine around the tcgen05 expert engine. The output, expert ids
and contributions must equal the one-GPU layer (k3xb_moe_layer_forward) bit
for bit: the per-token expert math does not depend on which rank or tile
runs it, and the combine keeps the slot order.

A world of one runs on any GPU box (NCCL sends to itself); the two-rank
test needs two GPUs and skips otherwise.
"""
import os

import numpy as np
import pytest

from gpu_util import layer_to_dev, to_dev, torch_cuda
from oracle import bf16_normal, make_moe_layer

pytestmark = pytest.mark.gpu

DIMS = dict(hidden=512, inter=256, experts=16, top_k=4, shared_inter=256)


def _layer(rs):
    d = DIMS
    return make_moe_layer(rs, 57, d["hidden"], d["inter"], d["experts"], d["top_k"], d["shared_inter"])


def _one_gpu(torch, ctx, layer, x):
    import k3xb
    d = layer_to_dev(torch, layer)
    desc = k3xb.moe_layer_desc(d, engine=k3xb.ENGINE_MXF4)
    T, H, K = x.shape[0], layer["hidden"], layer["top_k"]
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    con = torch.empty((T, K), dtype=torch.float32, device="cuda")
    ctx.moe_layer_forward(desc, to_dev(torch, x), out, ids, con)
    ctx.sync()
    return out.cpu().numpy(), ids.cpu().numpy(), con.cpu().numpy()


def _ep(torch, ctx, layer, x, rank, world):
    import k3xb
    d = layer_to_dev(torch, layer)
    local = k3xb.ep_local_layer(d, rank, world)
    desc = k3xb.moe_layer_desc(local, engine=k3xb.ENGINE_MXF4)
    T = x.shape[0] // world
    xr = to_dev(torch, x[rank * T:(rank + 1) * T])
    H, K = layer["hidden"], layer["top_k"]
    out = torch.empty((T, H), dtype=torch.float32, device="cuda")
    ids = torch.empty((T, K), dtype=torch.int32, device="cuda")
    con = torch.empty((T, K), dtype=torch.float32, device="cuda")
    ctx.ep_moe_layer_forward(desc, layer["experts"], xr, out, ids, con)
    ctx.sync()
    return out.cpu().numpy(), ids.cpu().numpy(), con.cpu().numpy()


def test_ep_world_of_one_equals_layer(rs):
    import k3xb
    torch = torch_cuda()
    layer = _layer(rs)
    x = bf16_normal(np.random.default_rng(58), (12, DIMS["hidden"]))
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        want = _one_gpu(torch, ctx, layer, x)
        ctx.ep_init(k3xb.ep_unique_id(), 0, 1)
        got = _ep(torch, ctx, layer, x, 0, 1)
        for g, w in zip(got, want):
            np.testing.assert_array_equal(g, w)
        ctx.ep_finalize()
    finally:
        ctx.close()


def _rank_main(rank, world, uid, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "project-k3x_b200"), os.path.join(root, "oracle")]
    import torch

    import k3xb
    from oracle import Restatement
    torch.cuda.set_device(rank)
    rs = Restatement()
    layer = _layer(rs)
    x = bf16_normal(np.random.default_rng(59), (8 * world, DIMS["hidden"]))
    ctx = k3xb.Context(rank)
    ctx.use_stream()
    ctx.ep_init(uid, rank, world)
    out, ids, con = _ep(torch, ctx, layer, x, rank, world)
    np.save(os.path.join(out_dir, f"out{rank}.npy"), out)
    np.save(os.path.join(out_dir, f"ids{rank}.npy"), ids)
    ctx.ep_finalize()
    ctx.close()


def test_ep_two_ranks_equal_one_gpu(rs, tmp_path):
    torch = torch_cuda()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    import k3xb
    world = 2
    uid = k3xb.ep_unique_id()
    mp.start_processes(_rank_main, args=(world, uid, str(tmp_path)), nprocs=world, start_method="spawn")
    layer = _layer(rs)
    x = bf16_normal(np.random.default_rng(59), (8 * world, DIMS["hidden"]))
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        want_out, want_ids, _ = _one_gpu(torch, ctx, layer, x)
    finally:
        ctx.close()
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"ids{r}.npy"), want_ids[r * 8:(r + 1) * 8])
        np.testing.assert_array_equal(np.load(tmp_path / f"out{r}.npy"), want_out[r * 8:(r + 1) * 8])

