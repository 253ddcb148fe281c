"""Expert-parallel MoE layer: the dispatch / local plan / return / combine
algorithm of csrc/ep.cu, restated on the CPU with the oracle's expert math
and run as 2 and 4 gloo ranks (experts split 4 and 2 per rank), for the
plain MoE and for LatentMoE (latent rows are projected on the home rank,
sent, computed and returned; the routed norm and up projection run at
home). Its output must equal the single-process oracle layer bit for bit
(the combine keeps the one-GPU slot order), which is the property the CUDA
path is tested for on 2 GPUs in test_gpu_ep.py / test_gpu_ep_verify.py and
with a world of one in test_gpu_latent.py.

The CUDA path stores into the other ranks' windows over peer memory. Here
each rank's stores are all-gathered (gloo has no one-sided puts) and every
rank keeps those addressed to it:
- dispatch: a token's metadata to every rank, its row (as bf16, exact for
  the bf16-valued rows) only to the ranks that own one of its experts; the
  rows a rank does not receive are NaN here, so a plan that read one would
  poison the output;
- return: each (token, slot) output row is stored by exactly one rank, the
  owner of the slot's expert, into the home rank's output region.
"""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import Restatement, bf16_normal, make_moe_layer

NO_ENTRY = 0xFFFFFFFF
DIMS = dict(hidden=256, inter=128, experts=8, top_k=3, shared_inter=128, tokens_per_rank=5)


def _layer(rs, latent=0):
    d = DIMS
    return make_moe_layer(rs, 91, d["hidden"], d["inter"], d["experts"], d["top_k"], d["shared_inter"],
                          latent=latent)


def _hidden(world):
    return bf16_normal(np.random.default_rng(92), (DIMS["tokens_per_rank"] * world, DIMS["hidden"]))


def _expert(rs, L, e, x):
    H, I = L.get("latent") or L["hidden"], L["inter"]   # the experts' width
    g = rs.mxfp4_matmul(x, L["gate_packed"][e], L["gate_scales"][e], I, H)
    u = rs.mxfp4_matmul(x, L["up_packed"][e], L["up_scales"][e], I, H)
    return rs.round_bf16(rs.mxfp4_matmul(rs.swiglu(g, u), L["down_packed"][e], L["down_scales"][e], H, I))


def _exchange(send, world):
    """send [world][...] -> recv [world][...] (recv[g] = rank g's send[me])."""
    me = dist.get_rank()
    send = np.ascontiguousarray(send)
    as_int = send.dtype == np.uint32   # gloo has no uint32: move the bits as int32
    t = torch.from_numpy(send.view(np.int32) if as_int else send)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t)
    recv = np.stack([p.numpy()[me] for p in parts])
    return recv.view(np.uint32) if as_int else recv


def _owner(E, world):
    """A placement (k3xb_ep_balance of a seeded load), or the ranges."""
    import k3xb
    return k3xb.ep_balance(np.random.default_rng(11).random(E).astype(np.float32), world)


def _ep_rank(rank, world, port, out_dir, latent, placed=False):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rs = Restatement()
    L = _layer(rs, latent)
    E, K, H = L["experts"], L["top_k"], L["hidden"]
    D = latent or H   # rows sent, computed and returned: latent rows for LatentMoE
    E_r, T = E // world, DIMS["tokens_per_rank"]
    owner = _owner(E, world) if placed else None

    def own(e):   # (rank, local index) holding expert e
        e = int(e)
        return (int(owner[e]) >> 16, int(owner[e]) & 0xFFFF) if owner is not None else divmod(e, E_r)
    expert_at = {own(e): e for e in range(E)}
    x_in = _hidden(world)[rank * T:(rank + 1) * T]
    # LatentMoE: the latent projection happens on the home rank (official_moe.cpp:296)
    x = np.stack([rs.bf16_matvec(x_in[t], L["routed_down"]) for t in range(T)]) if latent else x_in
    # route on the home rank (all E logits)
    ids = np.empty((T, K), np.uint32)
    con = np.empty((T, K), np.float32)
    for t in range(T):
        ids[t], con[t] = rs.route(x_in[t], L["router"], L["correction"], K)
    # dispatch: metadata (local expert << 8 | slot, or none) to every rank;
    # the row only where one of its slots' experts lives, as bf16 words
    meta = np.full((world, T, K), NO_ENTRY, np.uint32)
    for g in range(world):
        for t in range(T):
            for j in range(K):
                g_e, local = own(ids[t, j])
                if g_e == g:
                    meta[g, t, j] = local << 8 | j
    assert np.array_equal(rs.round_bf16(x), x)   # bf16-valued rows travel as bf16 exactly
    send_x = np.full((world, T, D), np.nan, np.float32)
    for g in range(world):
        for t in range(T):
            if (meta[g, t] != NO_ENTRY).any():
                send_x[g, t] = x[t]
    recv_meta = _exchange(meta, world)
    recv_x = _exchange(send_x, world)
    # local expert-major plan: ascending local expert, (row, slot) order
    rows = recv_x.reshape(world * T, D)
    m = recv_meta.reshape(world * T, K)
    put = np.full((world, T, K, D), np.nan, np.float32)   # stores addressed to each home rank
    for e in range(E_r):
        for r in range(world * T):
            for j in range(K):
                if m[r, j] != NO_ENTRY and (m[r, j] >> 8) == e:
                    home, t = divmod(r, T)
                    put[home, t, m[r, j] & 0xFF] = _expert(rs, L, expert_at[(rank, e)], rows[r])
    landed = _exchange(put, world)   # landed[g]: what rank g stored into this rank's region
    written = ~np.isnan(landed).all(axis=3)
    assert (written.sum(axis=0) == 1).all(), "every (token, slot) row is stored by exactly one rank"
    y_home = np.nansum(np.where(written[..., None], landed, 0.0), axis=0).astype(np.float32)
    # combine in slot order with each slot's owner (then, for LatentMoE, the
    # routed norm and up projection, :323-331), then + shared
    out = np.empty((T, H), np.float32)
    for t in range(T):
        ys = np.stack([y_home[t, j] for j in range(K)])
        mixed = rs.routed_combine(ys, con[t])
        if latent:
            mixed = rs.bf16_matvec(rs.rms_norm(mixed, L["routed_norm"], L["latent_eps"]), L["routed_up"])
        gs = rs.bf16_matvec(x_in[t], L["shared_gate"])
        us = rs.bf16_matvec(x_in[t], L["shared_up"])
        shared = rs.bf16_matvec(rs.swiglu(gs, us), L["shared_down"])
        out[t] = rs.round_bf16(mixed + shared)
    np.save(os.path.join(out_dir, f"out{rank}.npy"), out)
    np.save(os.path.join(out_dir, f"ids{rank}.npy"), ids)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world,latent,placed", [(2, 0, False), (2, 128, False), (4, 0, False), (4, 0, True),
                                                 (2, 128, True)])
def test_ep_restatement_equals_one_process(rs, tmp_path, world, latent, placed):
    port = 29500 + (os.getpid() + latent + 7 * world + 3 * placed) % 2000
    mp.start_processes(_ep_rank, args=(world, port, str(tmp_path), latent, placed), nprocs=world,
                       start_method="spawn")
    L = _layer(rs, latent)
    want, want_ids, _ = rs.moe_layer(L, _hidden(world))
    T = DIMS["tokens_per_rank"]
    for r in range(world):
        np.testing.assert_array_equal(np.load(tmp_path / f"ids{r}.npy"), want_ids[r * T:(r + 1) * T])
        np.testing.assert_array_equal(np.load(tmp_path / f"out{r}.npy"), want[r * T:(r + 1) * T])
