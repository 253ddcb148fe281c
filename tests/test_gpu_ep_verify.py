"""The expert-parallel verify step (k3xb_ep_verify_step) against the
one-GPU verify step (k3xb_verify_step), bit for bit: logits, accepted
counts, committed tokens and the committed KDA states, over several
consecutive steps (each step starts from the states the previous one
committed, and the exchange alternates its window halves).

With and without an expert placement (k3xb_moe_layer.ep_owner from
k3xb_ep_balance). Expert parallelism moves bf16-valued rows and bf16-rounded expert outputs,
and every per-token quantity is computed by the same kernels in the same
order whichever rank runs it, so equality is exact. A world of one runs on
any GPU box; the two-rank case needs two GPUs (one process per GPU) and
skips otherwise.
"""
import os

import numpy as np
import pytest

from gpu_util import to_dev, torch_cuda
from oracle import Restatement, bf16_words, make_layer

pytestmark = pytest.mark.gpu

DIMS = dict(hidden=256, heads=4, head_dim=64, experts=16, top_k=4, inter=128, shared_inter=128)
S_PER_RANK, DRAFTS, STEPS, V = 3, 4, 3, 1024


def _setup(rs, S):
    c = DIMS
    H, P = c["hidden"], c["heads"] * c["head_dim"]
    layers = [make_layer(rs, 70 + l, H, c["heads"], c["head_dim"], c["experts"], c["top_k"], c["inter"],
                         c["shared_inter"]) for l in range(2)]
    g = np.random.default_rng(71)
    emb = bf16_words(g.normal(0, 1.0, size=(V, H)))
    lm = bf16_words(g.normal(0, 0.02, size=(V, H)))
    fnorm = bf16_words(np.ones(H, np.float32))
    conv = np.stack([np.stack([np.stack([bf16_words(g.normal(0, 0.5, size=3 * P)) for _ in range(3)])
                               for _ in range(S)]) for _ in range(2)])
    rec = g.normal(0, 0.05, size=(2, S, c["heads"], c["head_dim"], c["head_dim"])).astype(np.float32)
    tokens = g.integers(0, V, size=(STEPS, S, DRAFTS + 1)).astype(np.int32)
    return layers, emb, lm, fnorm, conv, rec, tokens


def _owner(world):
    """An expert placement that is not the contiguous ranges (k3xb_ep_balance
    of a seeded load)."""
    import k3xb
    return k3xb.ep_balance(np.random.default_rng(17).random(DIMS["experts"]).astype(np.float32), world)


def _model(torch, layers, emb, lm, fnorm, rank=None, world=None, owner=None):
    import k3xb
    from test_gpu_draft import _layer_dev
    descs, keep = [], []
    for layer in layers:
        d = _layer_dev(torch, layer)
        if world is not None:
            d = dict(d, moe=k3xb.ep_local_layer(d["moe"], rank, world, owner=owner))
        keep.append(d)
        descs.append(k3xb.layer_desc(d))
    e, l, f = to_dev(torch, emb), to_dev(torch, lm), to_dev(torch, fnorm)
    return k3xb.verify_model_desc(descs, V, l, embedding=e, final_norm=f), (keep, e, l, f)


def _steps(torch, ctx, model, conv, rec, tokens, experts_total=None):
    """STEPS verify steps from (conv, rec); returns per step (logits,
    accepted, committed, count) and the final states."""
    import k3xb
    S = tokens.shape[1]
    conv_d, rec_d = to_dev(torch, conv), to_dev(torch, rec)
    out = []
    for i in range(STEPS):
        tok = to_dev(torch, tokens[i])
        drafts = to_dev(torch, np.ascontiguousarray(tokens[i][:, 1:]))
        logits = torch.empty((S, DRAFTS + 1, V), dtype=torch.float32, device="cuda")
        acc = torch.zeros(S, dtype=torch.int32, device="cuda")
        com = torch.zeros((S, DRAFTS + 1), dtype=torch.int32, device="cuda")
        cnt = torch.zeros(S, dtype=torch.int32, device="cuda")
        io = k3xb.verify_io_desc(S, DRAFTS, conv_d, rec_d, acc, com, cnt, drafts, tokens=tok, logits=logits)
        if experts_total is None:
            ctx.verify_step(model, io)
        else:
            ctx.ep_verify_step(model, io, experts_total)
        ctx.sync()
        out.append(tuple(t.cpu().numpy() for t in (logits, acc, com, cnt)))
    return out, conv_d.cpu().numpy(), rec_d.cpu().numpy()


def _assert_same(got, want, what):
    for i, (g, w) in enumerate(zip(got, want)):
        for name, a, b in zip(("logits", "accepted", "committed", "count"), g, w):
            np.testing.assert_array_equal(a, b, err_msg=f"{what}: step {i} {name}")


@pytest.mark.parametrize("placed", [False, True])
def test_ep_verify_world_of_one_equals_verify_step(rs, placed):
    import k3xb
    torch = torch_cuda()
    layers, emb, lm, fnorm, conv, rec, tokens = _setup(rs, S_PER_RANK)
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        model, keep = _model(torch, layers, emb, lm, fnorm)
        want, want_conv, want_rec = _steps(torch, ctx, model, conv, rec, tokens)
        ctx.ep_init(k3xb.ep_unique_id(), 0, 1)
        ep_model, ep_keep = _model(torch, layers, emb, lm, fnorm, 0, 1,
                                   owner=_owner(1) if placed else None)   # placed: a permuted stack
        got, got_conv, got_rec = _steps(torch, ctx, ep_model, conv, rec, tokens, DIMS["experts"])
        _assert_same(got, want, "world of one")
        np.testing.assert_array_equal(got_conv, want_conv)
        np.testing.assert_array_equal(got_rec, want_rec)
        assert ctx.stats()["moe_layer_calls"] > 0
        ctx.ep_finalize()
    finally:
        ctx.close()


def _rank_main(rank, world, uid, out_dir, placed=False):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(root, "project-k3x_b200"), os.path.join(root, "oracle"), os.path.join(root, "tests")]
    import torch

    import k3xb
    torch.cuda.set_device(rank)
    rs = Restatement()
    layers, emb, lm, fnorm, conv, rec, tokens = _setup(rs, S_PER_RANK * world)
    mine = slice(rank * S_PER_RANK, (rank + 1) * S_PER_RANK)
    ctx = k3xb.Context(rank)
    ctx.use_stream()
    ctx.ep_init(uid, rank, world)
    model, keep = _model(torch, layers, emb, lm, fnorm, rank, world, owner=_owner(world) if placed else None)
    got, got_conv, got_rec = _steps(torch, ctx, model, np.ascontiguousarray(conv[:, mine]),
                                    np.ascontiguousarray(rec[:, mine]), np.ascontiguousarray(tokens[:, mine]),
                                    DIMS["experts"])
    for i, step in enumerate(got):
        for name, a in zip(("logits", "accepted", "committed", "count"), step):
            np.save(os.path.join(out_dir, f"{name}{i}_{rank}.npy"), a)
    np.save(os.path.join(out_dir, f"conv_{rank}.npy"), got_conv)
    np.save(os.path.join(out_dir, f"rec_{rank}.npy"), got_rec)
    ctx.ep_finalize()
    ctx.close()


@pytest.mark.parametrize("placed", [False, True])
def test_ep_verify_two_ranks_equal_one_gpu(rs, tmp_path, placed):
    torch = torch_cuda()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp

    import k3xb
    world = 2
    uid = k3xb.ep_unique_id()
    mp.start_processes(_rank_main, args=(world, uid, str(tmp_path), placed), nprocs=world, start_method="spawn")
    layers, emb, lm, fnorm, conv, rec, tokens = _setup(rs, S_PER_RANK * world)
    ctx = k3xb.Context(0)
    ctx.use_stream()
    try:
        model, keep = _model(torch, layers, emb, lm, fnorm)
        want, want_conv, want_rec = _steps(torch, ctx, model, conv, rec, tokens)
    finally:
        ctx.close()
    for r in range(world):
        mine = slice(r * S_PER_RANK, (r + 1) * S_PER_RANK)
        got = [tuple(np.load(tmp_path / f"{name}{i}_{r}.npy") for name in ("logits", "accepted", "committed", "count"))
               for i in range(STEPS)]
        _assert_same(got, [tuple(a[mine] for a in step) for step in want], f"rank {r}")
        np.testing.assert_array_equal(np.load(tmp_path / f"conv_{r}.npy"), want_conv[:, mine])
        np.testing.assert_array_equal(np.load(tmp_path / f"rec_{r}.npy"), want_rec[:, mine])
